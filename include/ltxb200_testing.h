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

/* Force every (sample, head, 256-query) unit of the calling thread's subsequent
 * ltx_attention_ws calls (bf16, Tk > 128) to run as `parts` key-range parts merged by the
 * last one (1..8; parts = 1 runs each unit through the part kernel over all its keys),
 * 0 for the automatic plan, or -1 to never split. Shapes whose key tiles (Tk / 128, Tk
 * a multiple of 128) `parts` does not divide run unsplit. Thread-local;
 * ltx_attention_workspace_bytes follows it. */
 one thread waits on an mbarrier that nothing arrives on,
 * through the bounded wait of the tcgen05 kernels, for at most `limit_cycles` SM cycles
 * (<= 1e8, about 50 ms); it then gives up, sets bit 1 (wait timed out) of the device
 * error word that ltx_device_error_flags reads, writes 1 to the device int `returned`
 * (2 would mean the wait completed) and returns. The context stays usable. */
int ltx_test_attention_force_split(int parts);
/* The automatic split plan of one attention launch, host arithmetic only: for `units`
 * (sample, head, 256-query) units over Tk keys on `sms` SMs, the units that run whole
 * (*n_full) and the parts each remaining unit is split into (*split_k; 1: no split). */
int ltx_test_attention_plan(int64_t units, int64_t Tk, int sms, int* n_full, int* split_k);
int ltx_test_bounded_wait(unsigned long long limit_cycles, int* returned, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* LTXB200_TESTING_H */
