/*
 * Instantiates the reference's own single-header C decoder
 * (ref/c/hct_decoder.h in the haagenti repository) as a shared library so
 * the oracle tests can cross-check the IDCT against it.  Test
 * infrastructure only; compiled from the reference sources in place by
 * oracle/Makefile (target `ref`), output in oracle/_ref/.
 */
#define HCT_IMPLEMENTATION
#include "hct_decoder.h"
