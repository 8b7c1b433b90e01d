// Host build of the GPU Zstandard decoder (haagenti_b200/csrc/zstd_core.cuh
// compiles as plain C++ with one lane) checked against libzstd, the library
// the reference's `zstd` crate binds.  Run by tests/test_zstd_host.py.
//
// For every case: data of one of six kinds, compressed by libzstd (levels,
// checksums, content size on and off), then
//   * decode() must give libzstd's bytes;
//   * when the block-parallel plan accepts the frame, decoding its blocks
//     (decode_block, then decode_seq_blocks) must agree with decode() in
//     code, bytes and position;
//   * a few corrupted copies: decode() must fail wherever libzstd fails
//     (it may also fail where libzstd's fast Huffman path accepts a stream
//     that is not consumed exactly; those are counted, not failed).
// Prints one summary line; exit status 1 on any disagreement.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <vector>

#include "../haagenti_b200/csrc/zstd_core.cuh"

extern "C" {
size_t ZSTD_compressBound(size_t srcSize);
size_t ZSTD_decompress(void *dst, size_t dstCapacity, const void *src, size_t compressedSize);
unsigned ZSTD_isError(size_t code);
void *ZSTD_createCCtx(void);
size_t ZSTD_CCtx_setParameter(void *cctx, int param, int value);
size_t ZSTD_compress2(void *cctx, void *dst, size_t dstCapacity, const void *src, size_t srcSize);
size_t ZSTD_freeCCtx(void *cctx);
}

using namespace hct;

static int g_plan = 0, g_plan_ok = 0, g_stricter = 0;

static std::vector<uint8_t> make(int kind, size_t n, std::mt19937_64 &g) {
    std::vector<uint8_t> v(n);
    if (kind == 0) {  // random bytes
        for (auto &x : v) x = (uint8_t)g();
    } else if (kind == 1) {  // zeros
    } else if (kind == 2) {  // text
        const char *w[] = {"alpha ", "beta ", "gamma ", "delta ", "tensor ", "weight ", "zstd ", "block "};
        size_t i = 0;
        while (i < n) {
            const char *s = w[g() % 8];
            for (size_t k = 0; s[k] && i < n; k++) v[i++] = (uint8_t)s[k];
        }
    } else if (kind == 3) {  // fp16 N(0, 0.02)
        std::normal_distribution<float> d(0.f, 0.02f);
        for (size_t i = 0; i + 1 < n; i += 2) {
            const float f = d(g);
            uint32_t b;
            memcpy(&b, &f, 4);
            const uint32_t e = (b >> 23) & 0xff;
            uint16_t h = (uint16_t)((b >> 16) & 0x8000);
            if (e >= 113) h |= (uint16_t)(((e - 112) << 10) | ((b >> 13) & 0x3ff));
            v[i] = (uint8_t)h;
            v[i + 1] = (uint8_t)(h >> 8);
        }
    } else if (kind == 4) {  // ramp with noise
        for (size_t i = 0; i < n; i++) v[i] = (uint8_t)((i * 7 + (g() % 3 == 0 ? g() : 0)) & 0xff);
    } else {  // runs and noise
        for (size_t i = 0; i < n; i++) v[i] = (uint8_t)(i % 251 < 200 ? (i / 13) & 0xff : g());
    }
    return v;
}

static int check(const std::vector<uint8_t> &comp, const std::vector<uint8_t> &ref, bool ref_ok,
                 size_t cap, const char *tag) {
    zs::Workspace *ws = new zs::Workspace();
    std::vector<uint8_t> out(cap + 16), lit(zs::LIT_SCRATCH);
    uint64_t acc[4];
    const zs::Job job{comp.data(), comp.size(), out.data(), cap, lit.data()};
    const zs::Result r = zs::decode(ws, job, 0, 1, acc);
    const bool ok = r.code == zs::OK;
    int fails = 0;
    if (ok && !ref_ok) {
        printf("ACCEPTS %s: libzstd rejects\n", tag);
        fails++;
    } else if (!ok && ref_ok) {
        g_stricter++;
    } else if (ok && (r.written != ref.size() || (ref.size() && memcmp(out.data(), ref.data(), ref.size())))) {
        printf("BYTES %s\n", tag);
        fails++;
    }
    // the block-parallel path, where the plan takes the frame
    zs::JobPlan jp{0, ~0ull, 0, 0, 0, 0, 0, 0, 0};
    uint32_t cnt = 0;
    if (zs::plan_job(comp.data(), comp.size(), cap, 0, &jp, nullptr, &cnt)) {
        g_plan++;
        std::vector<zs::BlockDesc> d(cnt + 1);
        zs::plan_job(comp.data(), comp.size(), cap, 0, &jp, d.data(), &cnt);
        zs::HufWs *hw = new zs::HufWs();
        std::vector<uint8_t> po(cap + 16, 0xEE);
        bool all = true;
        for (uint32_t i = 0; i < cnt; i++)
            if (!(d[i].meta & zs::META_SEQ)) all = all && zs::decode_block(hw, comp.data(), d[i], po.data(), 0, 1);
        delete hw;
        jp.count = cnt;
        if (all && jp.nseq) {
            const zs::Job j2{comp.data(), comp.size(), po.data(), cap, lit.data()};
            all = zs::decode_seq_blocks(ws, j2, jp, d.data(), nullptr, 0, 1);
        }
        if (all) {
            g_plan_ok++;
            int code = zs::OK;
            if (jp.ckpos != ~0ull) {
                uint64_t a2[4];
                const uint64_t h = zs::xxh64(po.data(), jp.total, 0, 1, a2, nullptr);
                if ((uint32_t)h != zs::rd32(comp.data() + jp.ckpos)) code = zs::E_CHECKSUM;
            }
            if (code != r.code) {
                printf("PLAN CODE %s: %d vs %d\n", tag, code, r.code);
                fails++;
            } else if (code == zs::OK &&
                       (jp.total != r.written || jp.lastpos != r.pos ||
                        (jp.total && memcmp(po.data(), out.data(), jp.total)))) {
                printf("PLAN BYTES %s\n", tag);
                fails++;
            }
        }
    }
    delete ws;
    return fails;
}

int main() {
    std::mt19937_64 g(1234);
    int fails = 0, cases = 0;
    const size_t sizes[] = {0, 1, 5, 31, 100, 1000, 4096, 65536, 131072, 300000, 1000000};
    const int levels[] = {-5, 1, 3, 9, 19};
    for (int kind = 0; kind < 6; kind++)
        for (size_t n : sizes)
            for (int lv : levels)
                for (int ck = 0; ck < 2; ck++) {
                    if (n > 300000 && lv > 9) continue;
                    const auto data = make(kind, n, g);
                    void *cctx = ZSTD_createCCtx();
                    ZSTD_CCtx_setParameter(cctx, 100, lv);               // compression level
                    ZSTD_CCtx_setParameter(cctx, 201, ck);               // checksum flag
                    ZSTD_CCtx_setParameter(cctx, 200, (int)(n % 3 != 0)); // content size flag
                    std::vector<uint8_t> comp(ZSTD_compressBound(n) + 64);
                    const size_t c = ZSTD_compress2(cctx, comp.data(), comp.size(), data.data(), n);
                    ZSTD_freeCCtx(cctx);
                    if (ZSTD_isError(c)) {
                        printf("libzstd compress error\n");
                        return 2;
                    }
                    comp.resize(c);
                    char tag[128];
                    snprintf(tag, sizeof tag, "kind%d n%zu lv%d ck%d", kind, n, lv, ck);
                    cases++;
                    fails += check(comp, data, true, n + 1024, tag);
                    for (int t = 0; t < 2 && c > 8; t++) {  // corrupted copies
                        auto bad = comp;
                        const size_t at = 4 + g() % (c - 4);
                        bad[at] ^= (uint8_t)(1 + g() % 255);
                        std::vector<uint8_t> rb(n + 1024);
                        const size_t dn = ZSTD_decompress(rb.data(), rb.size(), bad.data(), bad.size());
                        const bool rok = !ZSTD_isError(dn);
                        if (rok) rb.resize(dn);
                        char tg[160];
                        snprintf(tg, sizeof tg, "%s corrupt@%zu", tag, at);
                        cases++;
                        fails += check(bad, rok ? rb : std::vector<uint8_t>(), rok, n + 1024, tg);
                    }
                }
    printf("cases %d failures %d stricter %d planned %d planned_decoded %d\n", cases, fails, g_stricter,
           g_plan, g_plan_ok);
    return fails != 0;
}
