// Row-sharded matvec with the all-gather of its output rows fused into the kernel, over NVLink peer memory.
//
// The reference drives one board; this is the multi-GPU form of its matvec (driver/matvec_fpga.h:29-33,
// fpga_matvec4) for matrices whose rows are split across GPUs: rank r owns rows [r * rows, (r + 1) * rows).
// Each rank runs the group-quantized matvec (stage_activations + stream_tile, so every output is bit-identical
// to the reference C) on its shard, and instead of writing its rows locally and handing them to an all-gather,
// every tile stores its finished rows directly into every rank's gathered-output buffer (peer mappings opened
// through CUDA IPC). Only plain stores and system-scope atomics cross NVLink: no peer loads and no NCCL call.
//
// The kernel is persistent (one CTA per resident slot, each owning a balanced block of rows) so that the costs
// paid once per CTA -- staging the activations, the fence that publishes its rows, one count on a local counter --
// are paid once per slot rather than once per tile. Completion: each CTA fences its stores at GPU scope and adds 1
// to this rank's CTA counter; the CTA that brings it to the grid size fences at system scope (cumulatively
// covering every CTA's stores it has synchronized with), adds 1 to every rank's arrival counter (one fence, then
// relaxed adds: together a release), and then holds the kernel open until its own arrival counter shows every
// rank's signal for this call, read last by an acquire load. So when the kernel ends on a rank, the whole gathered
// vector is in that rank's memory. A system-scope fence costs about 1.4 us on this path, an acquire load one load,
// so the wait ends with the load rather than a second fence. With one rank the end of the kernel publishes the rows
// and no fence is needed: the last CTA only advances the call counter.
//
// The gathered output is double-buffered by call parity: a rank may start call e + 1 (and write into a peer's
// buffer) while that peer still reads the output of call e, but it cannot reach call e + 2 before the peer has
// finished call e + 1's kernel, which its stream orders after its reads of call e's output. The call number lives on
// the device (each rank's kernel advances its own counter once every rank's rows have arrived), so every call has
// the same launch arguments and a sequence of calls can be captured in a CUDA graph.
//
// The wait is bounded (kGatherWaitNs of globaltimer, and kGatherSpin polls); when it runs out (a peer never ran
// its kernel) it sets the gather's error word, read by mvb_gather_error, and the kernel ends.
#include <stdio.h>
#include <string.h>

#include <vector>

#include "../../include/matvec_b200.h"
#include "matvec_kernels.cuh"
#include "mvb_runtime.h"

namespace mvb {

constexpr int kMaxRanks = kMaxGatherRanks;
constexpr long kGatherSpin = 1L << 26;
constexpr unsigned long long kGatherWaitNs = 2000000000ull;
// Head of each rank's buffer, before the two output buffers: [0] arrival counter, [1] error word, [2] CTA counter,
// [3] completed calls.
constexpr size_t kGatherHead = 256;

struct GatherParams {
    MatvecParams mv;            // this rank's shard (mv.out unused)
    float *out[kMaxRanks];      // every rank's gathered output buffer 0 (own included); buffer 1 follows obuf later
    size_t obuf;                // floats between a rank's two output buffers
    unsigned *arrive[kMaxRanks];  // every rank's arrival counter
    unsigned *done;             // this rank's CTA counter (back to 0 at the end of every call)
    unsigned *calls;            // this rank's completed calls (output parity, arrival target)
    int *err;                   // this rank's error word
    int world, rank, rows;
};

// Relaxed add; the system-scope fence before the first of them makes the group a release. (A release add per
// rank would order each add after the previous one's round trip over NVLink.)
__device__ __forceinline__ void red_relaxed_sys(unsigned *p, unsigned v) {
    asm volatile("red.relaxed.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Polling load; once it sees the value, an acquire load of the same word ends the wait.
__device__ __forceinline__ unsigned ld_relaxed_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Fences for the release / acquire patterns (fence + relaxed access); sequential consistency is not needed.
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

template <int FMT>
__global__ void __launch_bounds__(kThreads, MatvecMinBlocks<FMT>::value) gather_matvec_kernel(const GatherParams gp) {
    extern __shared__ __align__(16) uint8_t smem[];
    const MatvecSmem<32> sm(smem, gp.mv.n / 32);
    const unsigned call = *gp.calls;  // read by every CTA before the last one advances it
    const size_t base = (size_t)gp.rank * gp.rows + (call & 1) * gp.obuf;
    stage_activations<FMT, 32, kXQuantized>(gp.mv, sm);
    int r0, r1;
    cta_rows(gp.rows, blockIdx.x, gridDim.x, r0, r1);
    for (int row0 = r0; row0 < r1; row0 += gp.mv.rt) {
        stream_tile<FMT, 32>(gp.mv, sm, row0, min(gp.mv.rt, r1 - row0), [&](int row, float v) {
#pragma unroll
            for (int q = 0; q < kMaxRanks; q++)
                if (q < gp.world) gp.out[q][base + row] = v;
        });
        __syncthreads();  // the next tile rewrites the product buffer
    }
    if (gp.world > 1 && threadIdx.x < 32) fence_acq_rel_gpu();  // warp 0 stored every row of this CTA
    __syncthreads();
    if (threadIdx.x != 0) return;
    if (atomicAdd(gp.done, 1u) != gridDim.x - 1) return;
    // The last CTA of this rank: every CTA's rows are stored. Signal every rank, then wait for all of them.
    *gp.done = 0;
    if (gp.world == 1) {  // every CTA read the call number before it was counted
        *gp.calls = call + 1u;
        return;
    }
    const unsigned target = (call + 1u) * (unsigned)gp.world;  // every rank's signal of this call
    fence_acq_rel_sys();
#pragma unroll
    for (int q = 0; q < kMaxRanks; q++)
        if (q < gp.world) red_relaxed_sys(gp.arrive[q], 1u);
    const unsigned long long t0 = global_ns();
    for (long i = 0; i < kGatherSpin; i++) {
        if ((int)(ld_relaxed_sys(gp.arrive[gp.rank]) - target) >= 0) {
            ld_acquire_sys(gp.arrive[gp.rank]);
            *gp.calls = call + 1u;
            return;
        }
        if ((i & 63) == 63 && global_ns() - t0 > kGatherWaitNs) break;
    }
    atomicExch(gp.err, 1);
    *gp.calls = call + 1u;
}

struct Gather {
    int rank = 0, world = 0, rows = 0, tokens = 1;
    uint8_t *mem = nullptr;        // [kGatherHead | output 0 | output 1], each output tokens x rows * world fp32
    std::vector<uint8_t *> peer;   // every rank's `mem`, mapped here (own included)
    unsigned calls = 0;            // calls enqueued through this handle (whether an output exists yet)
};

static size_t out_bytes(const Gather *g) { return (size_t)g->tokens * g->rows * g->world * 4; }

}  // namespace mvb

using namespace mvb;

extern "C" int mvb_gather_handle_size(void) { return (int)sizeof(cudaIpcMemHandle_t); }

extern "C" void *mvb_gather_create_batch(int rank, int world, int rows, int tokens, void *handle) {
    if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world || rows < 1 || tokens < 1 || !handle) {
        set_error("mvb_gather_create: need 1 <= world <= %d, 0 <= rank < world, rows >= 1, tokens >= 1, a handle "
                  "buffer", kMaxRanks);
        return nullptr;
    }
    Gather *g = new Gather;
    g->rank = rank;
    g->world = world;
    g->rows = rows;
    g->tokens = tokens;
    const size_t bytes = kGatherHead + 2 * out_bytes(g);
    cudaError_t e = cudaMalloc(&g->mem, bytes);
    if (e == cudaSuccess) e = cudaMemset(g->mem, 0, bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t *>(handle), g->mem);
    if (e != cudaSuccess) {
        set_error("mvb_gather_create: %s", cudaGetErrorString(e));
        if (g->mem) cudaFree(g->mem);
        delete g;
        return nullptr;
    }
    g->peer.assign(world, nullptr);
    g->peer[rank] = g->mem;
    return g;
}

extern "C" void *mvb_gather_create(int rank, int world, int rows, void *handle) {
    return mvb_gather_create_batch(rank, world, rows, 1, handle);
}

extern "C" int mvb_gather_connect(void *gather, const void *handles) {
    Gather *g = static_cast<Gather *>(gather);
    if (!g || !handles) {
        set_error("mvb_gather_connect: null argument");
        return -1;
    }
    const cudaIpcMemHandle_t *h = static_cast<const cudaIpcMemHandle_t *>(handles);
    for (int q = 0; q < g->world; q++) {
        if (q == g->rank || g->peer[q]) continue;
        void *p = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&p, h[q], cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            set_error("mvb_gather_connect: cannot map rank %d's buffer: %s", q, cudaGetErrorString(e));
            return -1;
        }
        g->peer[q] = static_cast<uint8_t *>(p);
    }
    return 0;
}

extern "C" int mvb_gather_matvec4(void *gather, const void *w, const void *ws, const void *xq, const void *xs, int n,
                                  int wbits, void *stream) {
    Gather *g = static_cast<Gather *>(gather);
    if (!g) {
        set_error("mvb_gather_matvec4: null gather");
        return -1;
    }
    for (int q = 0; q < g->world; q++)
        if (!g->peer[q]) {
            set_error("mvb_gather_matvec4: rank %d's buffer is not mapped (call mvb_gather_connect)", q);
            return -1;
        }
    if ((wbits != 4 && wbits != 8) || n <= 0 || n > kMaxN || n % 32) {
        set_error("mvb_gather_matvec4: unsupported n=%d wbits=%d (need wbits 4 or 8, n %% 32 == 0, n <= %d)", n,
                  wbits, kMaxN);
        return -1;
    }
    if (!w || !ws || !xq || !xs || ((uintptr_t)w & 15) || ((uintptr_t)xq & 15) || ((uintptr_t)ws & 1) ||
        ((uintptr_t)xs & 3)) {
        set_error("mvb_gather_matvec4: null or misaligned pointer");
        return -1;
    }
    GatherParams gp = {};
    MatvecParams &p = gp.mv;
    p.w = static_cast<const uint8_t *>(w);
    p.ws = ws;
    p.xq = static_cast<const int8_t *>(xq);
    p.xs = static_cast<const float *>(xs);
    p.n = n;
    p.d = g->rows;
    p.xmode = kXQuantized;
    const void *kernel = wbits == 4 ? (const void *)gather_matvec_kernel<kQ4F16> : (const void *)gather_matvec_kernel<kQ8F16>;
    size_t smem = 0;
    const int grid = row_layout(kernel, n, 32, g->rows, p.rt, smem);
    for (int q = 0; q < g->world; q++) {
        gp.out[q] = reinterpret_cast<float *>(g->peer[q] + kGatherHead);
        gp.arrive[q] = reinterpret_cast<unsigned *>(g->peer[q]);
    }
    gp.obuf = out_bytes(g) / 4;
    unsigned *head = reinterpret_cast<unsigned *>(g->mem);
    gp.err = reinterpret_cast<int *>(head + 1);
    gp.done = head + 2;
    gp.calls = head + 3;
    gp.world = g->world;
    gp.rank = g->rank;
    gp.rows = g->rows;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (wbits == 4) gather_matvec_kernel<kQ4F16><<<grid, kThreads, smem, s>>>(gp);
    else gather_matvec_kernel<kQ8F16><<<grid, kThreads, smem, s>>>(gp);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_error("mvb_gather_matvec4: launch failed: %s", cudaGetErrorString(e));
        return -1;
    }
    g->calls++;
    return 0;
}

// The batched form: m tokens through this rank's rows on the tensor cores (gemm.cu), every row stored into
// every rank's token-major gathered output (m x rows * world fp32) by the matmul's epilogue, completion signalled
// the same way.
extern "C" int mvb_gather_gemm4(void *gather, const void *w, const void *ws, const void *xq, const float *xs, int n,
                                int m, int ldx, int wbits, void *stream) {
    Gather *g = static_cast<Gather *>(gather);
    if (!g) {
        set_error("mvb_gather_gemm4: null gather");
        return -1;
    }
    for (int q = 0; q < g->world; q++)
        if (!g->peer[q]) {
            set_error("mvb_gather_gemm4: rank %d's buffer is not mapped (call mvb_gather_connect)", q);
            return -1;
        }
    if (m < 1 || m > g->tokens) {
        set_error("mvb_gather_gemm4: %d tokens, the gather holds at most %d", m, g->tokens);
        return -1;
    }
    PeerTargets pt = {};
    for (int q = 0; q < g->world; q++) {
        pt.out[q] = reinterpret_cast<float *>(g->peer[q] + kGatherHead);
        pt.arrive[q] = reinterpret_cast<unsigned *>(g->peer[q]);
    }
    pt.obuf = out_bytes(g) / 4;
    unsigned *head = reinterpret_cast<unsigned *>(g->mem);
    pt.err = reinterpret_cast<int *>(head + 1);
    pt.done = head + 2;
    pt.calls = head + 3;
    pt.world = g->world;
    pt.rank = g->rank;
    pt.col0 = g->rank * g->rows;
    if (gemm_launch(w, ws, xq, xs, nullptr, n, g->rows, m, ldx, g->rows * g->world, wbits,
                    static_cast<cudaStream_t>(stream), &pt))
        return -1;
    g->calls++;
    return 0;
}

// The output buffer of the last completed call, from the device's call counter (graph replays advance it without
// the host seeing the calls): synchronous, so read it once the calls' stream has finished.
extern "C" float *mvb_gather_output(void *gather) {
    Gather *g = static_cast<Gather *>(gather);
    if (!g || !g->calls) return nullptr;
    unsigned done = 0;
    if (cudaMemcpy(&done, g->mem + 12, 4, cudaMemcpyDeviceToHost) != cudaSuccess || !done) return nullptr;
    return reinterpret_cast<float *>(g->mem + kGatherHead + ((done - 1) & 1) * out_bytes(g));
}

extern "C" int mvb_gather_error(void *gather, void *stream) {
    Gather *g = static_cast<Gather *>(gather);
    if (!g) return -1;
    int v = 0;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (cudaMemcpyAsync(&v, g->mem + 4, 4, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return -1;
    return v;
}

extern "C" void mvb_gather_destroy(void *gather) {
    Gather *g = static_cast<Gather *>(gather);
    if (!g) return;
    cudaDeviceSynchronize();
    for (int q = 0; q < g->world; q++)
        if (q != g->rank && g->peer[q]) cudaIpcCloseMemHandle(g->peer[q]);
    if (g->mem) cudaFree(g->mem);
    delete g;
}
