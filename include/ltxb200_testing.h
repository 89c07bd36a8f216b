/*
 * ltxb200_testing.h - test hooks of libltxb200.so. Not part of the stable C ABI in
 * ltxb200.h: they exist so the parity tests can force one code path of a kernel family
 * and compare it with another. No counterpart in the reference.
 */
#ifndef LTXB200_TESTING_H
#define LTXB200_TESTING_H

#ifdef __cplusplus
extern "C" {
#endif

/* Force single-CTA tcgen05 GEMM tiles of 128 or 256 columns for the calling thread's
 * subsequent ltx_linear calls, or 0 for the automatic choice (256-column tiles computed
 * by CTA pairs when N >= 512 and M >= 256). The setting is thread-local: other threads'
 * GEMMs are not affected. Every choice gives bit-identical results. */
int ltx_gemm_set_tile_n(int bn);

#ifdef __cplusplus
}
#endif
#endif /* LTXB200_TESTING_H */
