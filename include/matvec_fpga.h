/* Drop-in replacement for the reference's board driver API (driver/matvec_fpga.h:12-33), served by
 * libmatvec_b200.so on an NVIDIA B200. The six declarations below keep the reference's names, argument
 * meanings, return conventions and error behaviour, so qwen/qwen.c and runq/runq.c compile with -DFPGA against
 * this header and link -lmatvec_b200 without a single source change.
 *
 * What a "physical address" is here: fpga_alloc() returns a pinned host buffer and stores in *phys the CUDA
 * device address of its twin in HBM. Callers may add any byte offset to *phys (they carve matrices and vectors
 * out of big buffers) and pass the sum to fpga_matvec()/fpga_matvec4(). At each call the library maps every
 * address back to its buffer and moves data between the host buffer and its twin:
 *   - w/wq and ws ranges are weights: uploaded on first use and then treated as read-only. Hosts write every
 *     weight before their first matvec (qwen.c:324-329, runq.c:359-366); a weight range rewritten after it was
 *     first used is not seen again.
 *   - xq and xs are read from the host buffer on every call (they travel inside the kernel launch's parameters);
 *     the kernel writes out straight into the host buffer before the call returns (the device addresses the
 *     pinned buffer directly).
 * Every call is synchronous and waits at most MATVEC_TIMEOUT_S seconds (default 5, like the reference's
 * TIMEOUT_S, driver/matvec_fpga.cpp:34). After a call that timed out, every later matvec call returns -1 until
 * fpga_close(): that call's result copy may still be in flight. Not thread-safe, like the reference (one caller
 * thread). A call returns when the kernel's last CTA has written the call's number into a completion word in
 * mapped host memory (after the output, with a system-scope fence between); the host polls that word and asks
 * the stream about errors every 1024 polls. MATVEC_STATS=1 makes fpga_close() print the mean per-call times
 * (host enqueue, upload, kernel, download, completion wait, host time between calls) as one "matvec stats: {...}"
 * line on stderr.
 */
#ifndef MATVEC_FPGA_H
#define MATVEC_FPGA_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Replaces fpga_open (driver/matvec_fpga.h:15). Selects the CUDA device given by env FPGA_MEMIDX (default 0;
 * the reference's memory-bank index becomes the device ordinal) and creates the library's stream.
 * Idempotent. Returns 0, or -1 with a message on stderr. */
int fpga_open(void);

/* Replaces fpga_alloc (driver/matvec_fpga.h:19). Allocates `bytes` of pinned host memory (page aligned, zeroed)
 * and a device twin of the same size; returns the host pointer and stores the device address in *phys.
 * Kept until fpga_close(). NULL with a message on stderr on failure. */
void *fpga_alloc(size_t bytes, uint64_t *phys);

/* Replaces fpga_alloc_try (driver/matvec_fpga.h:22): same as fpga_alloc but silent on failure, for callers that
 * retry with a smaller size. Env MATVEC_ALLOC_LIMIT (bytes) makes it fail once that many bytes are allocated,
 * to exercise those callers' fallback paths. */
void *fpga_alloc_try(size_t bytes, uint64_t *phys);

/* Replaces fpga_matvec (driver/matvec_fpga.h:26; contract hls/matvec.h:1-19, runq.c matmul):
 *   out[i] = sum over g of ((float)(sum_{k<gs} wq[i*n + g*gs + k] * xq[g*gs + k]) * ws[(i*n)/gs + g]) * xs[g]
 * int8 weights, fp32 weight scales, group size gs in {32, 64}; groups added in order, bit-exact with runq.c.
 * Rejects gs not 32/64, n <= 0, n > 8192, n % gs != 0, d <= 0 (the reference's checks), an address outside every
 * buffer, or fp32 arrays ws/xs/out off their 4-byte alignment. wq and xq may sit at any byte address, as in the
 * reference (a misaligned range is read from an aligned device copy). Returns 0, or -1 with a message on stderr. */
int fpga_matvec(uint64_t wq, uint64_t ws, uint64_t xq, uint64_t xs, uint64_t out, int n, int d, int gs);

/* Replaces fpga_matvec4 (driver/matvec_fpga.h:30; contract hls4/matvec4.h:1-21, qwen.c matmul_cpu):
 *   out[i] = sum over g of ((float)(sum_{k<32} w[i*n + g*32 + k] * xq[g*32 + k]) * f16(ws[(i*n)/32 + g])) * xs[g]
 * wbits 4 (two's complement nibbles, element 2i low) or 8 (int8); fp16 scales; groups added in order,
 * bit-exact with qwen.c. Rejects wbits not 4/8, n <= 0, n > 8192, n % 32 != 0, d <= 0, any address not 64-byte
 * aligned, or an address outside every buffer. Returns 0, or -1 with a message on stderr. */
int fpga_matvec4(uint64_t w, uint64_t ws, uint64_t xq, uint64_t xs, uint64_t out, int n, int d, int wbits);

/* Replaces fpga_close (driver/matvec_fpga.h:33): frees every buffer and the stream. Safe when nothing is open. */
void fpga_close(void);

#ifdef __cplusplus
}
#endif
#endif
