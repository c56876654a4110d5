// Shared host-side helpers of libmatvec_b200.so: error reporting and the matvec launchers.
#pragma once
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stddef.h>
#include <stdint.h>

namespace mvb {

// Records the message for mvb_last_error() and prints it on stderr (the reference's drivers report there).
void set_error(const char *fmt, ...) __attribute__((format(printf, 1, 2)));
void clear_error();

// The unique ID of the calling thread's current CUDA context (cuCtxGetId: never reused within a process, so a
// context made after a cudaDeviceReset() has a new one), or 0 when there is no current context or the driver entry
// points are missing. Caches of device addresses are keyed by it.
unsigned long long current_context_id();

// Validates and launches one matvec. fmt: WeightFormat; gs: 32 or 64; xmode: XMode. pdl: launch with
// programmatic dependent launch. Returns 0, or -1 after set_error(). `who` prefixes messages.
int launch_matvec(const char *who, int fmt, int gs, const void *w, const void *ws, const void *xq, const void *xs,
                  const float *x, float *out, int n, int d, int xmode, cudaStream_t stream, bool pdl = false);

// One synchronous-style call of the drop-in driver (fpga_matvec / fpga_matvec4): activations xq_host (n int8) and
// xs_host (n/gs fp32) in host memory are copied into the launch's parameters; the kernel writes its rows to `out`
// (device) and its last CTA copies them to host_out (pinned host memory the device addresses), then writes seq into
// the mapped host word flag (device address), after a system-scope fence. done: a zeroed device counter (the kernel
// resets it). Inputs up to kCallSmallN columns travel in a 1 KB parameter block, larger ones in a kMaxN one. 0, or
// -1 after set_error().
constexpr int kCallSmallN = 1024;
int launch_matvec_call(const char *who, int fmt, int gs, const void *w, const void *ws, const int8_t *xq_host,
                       const float *xs_host, float *out, float *host_out, unsigned *done, unsigned *flag,
                       unsigned seq, int n, int d, cudaStream_t stream);

// Persistent row layout of a matvec kernel (matvec_kernels.cuh): returns the grid, sets the tile rows and the
// dynamic shared memory. resident_slots: resident CTAs of a kernel (blocks of `threads`) over all SMs of the
// current device.
int row_layout(const void *kernel, int n, int gs, int d, int &rt, size_t &smem);
int resident_slots(const void *kernel, size_t smem, int threads = 256);
int rows_per_tile(int n, int d);

// Where a row-sharded matmul stores its rows and how it signals completion (gather.cu's protocol): every rank's
// gathered output buffer 0 (token-major, ldo floats per token, this rank's rows at columns col0 ..; buffer 1 follows
// obuf floats later), every rank's arrival counter, this rank's CTA counter, call counter and error word. The call
// counter, kept on the device and advanced by the kernel itself, picks the output buffer (call parity) and the
// arrival count that means every rank has signalled this call, so the launch's arguments are the same for every
// call (a sequence of calls can be captured in a CUDA graph and replayed).
constexpr int kMaxGatherRanks = 8;
struct PeerTargets {
    float *out[kMaxGatherRanks];
    size_t obuf;
    unsigned *arrive[kMaxGatherRanks];
    unsigned *done;
    unsigned *calls;
    int *err;
    int world, rank, col0;
};

// The tensor-core prefill matmul of gemm.cu (mvb_gemm4) with an output leading dimension: out[t * ldo + i]. With
// peers, the rows go to every rank's gathered output instead and the call signals completion (the all-gather of a
// row-sharded matmul fused into it); out is then unused.
int gemm_launch(const void *w, const void *ws, const void *xq, const float *xs, float *out, int n, int d, int m, int ldx,
                int ldo, int wbits, cudaStream_t stream, const PeerTargets *peers = nullptr);

}  // namespace mvb
