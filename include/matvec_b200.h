/* Entry points of libmatvec_b200.so beyond the reference's six (include/matvec_fpga.h). None of these has a
 * counterpart in driver/matvec_fpga.h; the unchanged reference hosts never call them. They take CUDA device
 * pointers and a CUDA stream of the current device (as void *; NULL = CUDA's default stream), run
 * asynchronously and return 0, or -1 with the reason in mvb_last_error() (and on stderr).
 *
 * The arithmetic of every matvec here is the reference's (qwen.c:436-456, runq.c:430-458): int32 group sums,
 * p = ((float)isum * wscale) * xscale, groups added in order. Outputs are bit-identical to the reference C.
 */
#ifndef MATVEC_B200_H
#define MATVEC_B200_H
#include <stddef.h>
#include <stdint.h>
#include "matvec_fpga.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Text of the last error raised by any entry point of this library ("" if none). */
const char *mvb_last_error(void);

/* fpga_matvec4's computation on device pointers (the qwen path, hls4/matvec4.h:1-21): w (d*n*wbits/8 bytes),
 * ws (d*n/32 fp16), xq (n int8), xs (n/32 fp32) -> out (d fp32). wbits 4 or 8, n % 32 == 0, n <= 8192, d >= 1;
 * w and xq 16-byte aligned, ws 2-byte, xs and out 4-byte aligned. */
int mvb_matvec4(const void *w, const void *ws, const void *xq, const void *xs, float *out, int n, int d, int wbits,
                void *stream);

/* fpga_matvec's computation on device pointers (the runq path, hls/matvec.h:1-19): wq (d*n int8), ws (d*n/gs
 * fp32), xq (n int8), xs (n/gs fp32) -> out (d fp32). gs 32 or 64, n % gs == 0, n <= 8192, d >= 1;
 * wq and xq 16-byte aligned, ws/xs/out 4-byte aligned. */
int mvb_matvec(const void *wq, const void *ws, const void *xq, const void *xs, float *out, int n, int d, int gs,
               void *stream);

/* mvb_matvec4 with the activation quantization fused into the kernel's prologue: x is n fp32 values, quantized
 * per group of 32 exactly like qwen.c's quantize() (qwen.c:355-364) inside every CTA. x 16-byte aligned. */
int mvb_qmatvec4(const void *w, const void *ws, const float *x, float *out, int n, int d, int wbits, void *stream);

/* mvb_matvec with runq.c's quantize() (runq.c:244-270) fused into the prologue. x 16-byte aligned. */
int mvb_qmatvec(const void *wq, const void *ws, const float *x, float *out, int n, int d, int gs, void *stream);

/* Rows per CTA tile that the launchers pick for a d x n matrix (exposed for the benchmark's accounting). */
int mvb_rows_per_tile(int n, int d);

#ifdef __cplusplus
}
#endif
#endif
