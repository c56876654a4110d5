// Launchers of the matvec kernels and the device-pointer entry points of include/matvec_b200.h.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <map>
#include <mutex>
#include <tuple>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "../../include/matvec_b200.h"
#include "matvec_kernels.cuh"
#include "mvb_runtime.h"

namespace mvb {

static thread_local char g_err[512];

void set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
    fprintf(stderr, "%s\n", g_err);
}

void clear_error() { g_err[0] = 0; }

const char *last_error() { return g_err; }

unsigned long long current_context_id() {
    static std::once_flag once;
    static PFN_cuCtxGetCurrent_v4000 get_current = nullptr;
    static PFN_cuCtxGetId_v12000 get_id = nullptr;
    std::call_once(once, [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(f);
        f = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(f);
    });
    CUcontext c = nullptr;
    unsigned long long id = 0;
    if (!get_current || !get_id || get_current(&c) != CUDA_SUCCESS || !c || get_id(c, &id) != CUDA_SUCCESS) return 0;
    return id;
}

// Resident CTAs of `kernel` on the current device at kThreads threads and `smem` bytes (all SMs), cached per
// device, kernel and size; 148 * 4 if the device cannot be queried.
int resident_slots(const void *kernel, size_t smem, int threads) {
    static std::mutex mu;
    static std::map<std::tuple<int, const void *, size_t, int>, int> cache;
    const int fallback = threads == kThreads ? 148 * 4 : 148;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return fallback;
    std::lock_guard<std::mutex> lock(mu);
    const auto key = std::make_tuple(dev, kernel, smem, threads);
    const auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    int sms = 0, per_sm = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess || sms <= 0 ||
        per_sm <= 0) {
        cudaGetLastError();
        return fallback;  // not cached: a later call (say, once the kernel may take more shared memory) asks again
    }
    return cache[key] = sms * per_sm;
}

// Persistent row layout for d rows of n columns: one CTA per resident slot (at most one per row), each owning a
// balanced block of rows that it streams in tiles of rt <= 32 rows (one warp folds a tile). Returns the grid.
int row_layout(const void *kernel, int n, int gs, int d, int &rt, size_t &smem) {
    const int slots = resident_slots(kernel, matvec_smem_bytes(n, gs, 32));
    const int grid = d < slots ? d : slots;
    const int per_cta = (d + grid - 1) / grid;
    rt = per_cta < 32 ? per_cta : 32;
    smem = matvec_smem_bytes(n, gs, rt);
    return grid;
}

int rows_per_tile(int n, int d) {
    int rt = 1;
    size_t smem = 0;
    row_layout((const void *)matvec_kernel<kQ4F16, 32, kXQuantized>, n, 32, d, rt, smem);
    return rt;
}

template <int FMT, int GS, int XM>
static cudaError_t launch(MatvecParams p, cudaStream_t stream, bool pdl) {
    size_t smem = 0;
    const int grid = row_layout((const void *)matvec_kernel<FMT, GS, XM>, p.n, GS, p.d, p.rt, smem);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    if (pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return cudaLaunchKernelEx(&cfg, matvec_kernel<FMT, GS, XM>, p);
}

static bool aligned(const void *p, uintptr_t a) { return ((uintptr_t)p & (a - 1)) == 0; }

// Launches `kernel` with one argument by value (which may exceed 4 KB) on `grid` CTAs of kThreads.
template <typename K, typename A>
static cudaError_t cudaLaunchKernelEx_helper(K kernel, int grid, size_t smem, cudaStream_t stream, const A &arg) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    return cudaLaunchKernelEx(&cfg, kernel, arg);
}

int launch_matvec(const char *who, int fmt, int gs, const void *w, const void *ws, const void *xq, const void *xs,
                  const float *x, float *out, int n, int d, int xmode, cudaStream_t stream, bool pdl) {
    const bool quantized = xmode == kXQuantized;
    if (!((fmt == kQ8F32 && (gs == 32 || gs == 64)) || ((fmt == kQ4F16 || fmt == kQ8F16) && gs == 32))) {
        set_error("%s: unsupported format %d with group size %d", who, fmt, gs);
        return -1;
    }
    if (n <= 0 || n > kMaxN || n % gs || d <= 0) {
        set_error("%s: unsupported n=%d d=%d gs=%d (need n %% gs == 0, 0 < n <= %d, d >= 1)", who, n, d, gs, kMaxN);
        return -1;
    }
    if (!w || !ws || !out || (quantized ? (!xq || !xs) : !x)) {
        set_error("%s: null pointer argument", who);
        return -1;
    }
    if (!aligned(w, 16) || !aligned(ws, fmt == kQ8F32 ? 4 : 2) || !aligned(out, 4) ||
        (quantized ? (!aligned(xq, 16) || !aligned(xs, 4)) : !aligned(x, 16))) {
        set_error("%s: misaligned pointer (weights and int8 activations need 16 bytes, fp32 activations 16, "
                  "scales and out their element size)", who);
        return -1;
    }
    // The activation quantizer goes with the weight format: qwen.c's for the .qwb formats, runq.c's for runq's.
    if (!quantized && xmode != (fmt == kQ8F32 ? kXQuantizeRunq : kXQuantizeQwen)) {
        set_error("%s: activation mode %d does not go with weight format %d", who, xmode, fmt);
        return -1;
    }
    MatvecParams p;
    p.w = static_cast<const uint8_t *>(w);
    p.ws = ws;
    p.xq = static_cast<const int8_t *>(xq);
    p.xs = static_cast<const float *>(xs);
    p.x = x;
    p.out = out;
    p.n = n;
    p.d = d;
    p.xmode = xmode;
    cudaError_t e;
    if (fmt == kQ4F16) e = quantized ? launch<kQ4F16, 32, kXQuantized>(p, stream, pdl)
                                     : launch<kQ4F16, 32, kXQuantizeQwen>(p, stream, pdl);
    else if (fmt == kQ8F16) e = quantized ? launch<kQ8F16, 32, kXQuantized>(p, stream, pdl)
                                          : launch<kQ8F16, 32, kXQuantizeQwen>(p, stream, pdl);
    else if (gs == 32) e = quantized ? launch<kQ8F32, 32, kXQuantized>(p, stream, pdl)
                                     : launch<kQ8F32, 32, kXQuantizeRunq>(p, stream, pdl);
    else e = quantized ? launch<kQ8F32, 64, kXQuantized>(p, stream, pdl)
                       : launch<kQ8F32, 64, kXQuantizeRunq>(p, stream, pdl);
    if (e != cudaSuccess) {
        set_error("%s: kernel launch failed: %s", who, cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

// The call's layout: one CTA per 32 rows, up to the resident slots (row_layout's one CTA per slot would have every
// CTA of a small matrix stage the activations for one or two rows).
template <int FMT, int GS, int NMAX>
static cudaError_t launch_call(const MatvecParams &p, const int8_t *xq_host, const float *xs_host, float *host_out,
                               unsigned *done, unsigned *flag, unsigned seq, cudaStream_t stream) {
    CallArgs<NMAX, GS> a;
    a.p = p;
    a.host_out = host_out;
    a.done = done;
    a.flag = flag;
    a.seq = seq;
    memcpy(a.xq, xq_host, p.n);
    memcpy(a.xs, xs_host, (size_t)(p.n / GS) * 4);
    const int slots = resident_slots((const void *)matvec_call_kernel<FMT, GS, NMAX>, matvec_smem_bytes(p.n, GS, 32));
    const int tiles = (p.d + 31) / 32;
    const int grid = tiles < slots ? tiles : slots;
    const int per_cta = (p.d + grid - 1) / grid;
    a.p.rt = per_cta < 32 ? per_cta : 32;
    return cudaLaunchKernelEx_helper(matvec_call_kernel<FMT, GS, NMAX>, grid, matvec_smem_bytes(p.n, GS, a.p.rt),
                                     stream, a);
}

int launch_matvec_call(const char *who, int fmt, int gs, const void *w, const void *ws, const int8_t *xq_host,
                       const float *xs_host, float *out, float *host_out, unsigned *done, unsigned *flag,
                       unsigned seq, int n, int d, cudaStream_t stream) {
    if (!((fmt == kQ8F32 && (gs == 32 || gs == 64)) || ((fmt == kQ4F16 || fmt == kQ8F16) && gs == 32)) || n <= 0 ||
        n > kMaxN || n % gs || d <= 0 || !w || !ws || !out || !host_out || !done || !flag || !aligned(w, 16) ||
        !aligned(ws, fmt == kQ8F32 ? 4 : 2) || !aligned(out, 4) || !aligned(host_out, 4)) {
        set_error("%s: bad call (format %d, group size %d, n=%d, d=%d, or a null or misaligned pointer)", who, fmt, gs,
                  n, d);
        return -1;
    }
    MatvecParams p = {};
    p.w = static_cast<const uint8_t *>(w);
    p.ws = ws;
    p.out = out;
    p.n = n;
    p.d = d;
    p.xmode = kXQuantized;
    const bool small = n <= kCallSmallN;
    cudaError_t e;
    if (fmt == kQ4F16)
        e = small ? launch_call<kQ4F16, 32, kCallSmallN>(p, xq_host, xs_host, host_out, done, flag, seq, stream)
                  : launch_call<kQ4F16, 32, kMaxN>(p, xq_host, xs_host, host_out, done, flag, seq, stream);
    else if (fmt == kQ8F16)
        e = small ? launch_call<kQ8F16, 32, kCallSmallN>(p, xq_host, xs_host, host_out, done, flag, seq, stream)
                  : launch_call<kQ8F16, 32, kMaxN>(p, xq_host, xs_host, host_out, done, flag, seq, stream);
    else if (gs == 32)
        e = small ? launch_call<kQ8F32, 32, kCallSmallN>(p, xq_host, xs_host, host_out, done, flag, seq, stream)
                  : launch_call<kQ8F32, 32, kMaxN>(p, xq_host, xs_host, host_out, done, flag, seq, stream);
    else
        e = small ? launch_call<kQ8F32, 64, kCallSmallN>(p, xq_host, xs_host, host_out, done, flag, seq, stream)
                  : launch_call<kQ8F32, 64, kMaxN>(p, xq_host, xs_host, host_out, done, flag, seq, stream);
    if (e != cudaSuccess) {
        set_error("%s: kernel launch failed: %s", who, cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

}  // namespace mvb

using namespace mvb;

extern "C" const char *mvb_last_error(void) { return mvb::last_error(); }

extern "C" int mvb_rows_per_tile(int n, int d) { return rows_per_tile(n, d); }

extern "C" int mvb_matvec4(const void *w, const void *ws, const void *xq, const void *xs, float *out, int n, int d,
                           int wbits, void *stream) {
    if (wbits != 4 && wbits != 8) {
        set_error("mvb_matvec4: unsupported wbits=%d (need 4 or 8)", wbits);
        return -1;
    }
    return launch_matvec("mvb_matvec4", wbits == 4 ? kQ4F16 : kQ8F16, 32, w, ws, xq, xs, nullptr, out, n, d,
                         kXQuantized, static_cast<cudaStream_t>(stream));
}

extern "C" int mvb_matvec(const void *wq, const void *ws, const void *xq, const void *xs, float *out, int n, int d,
                          int gs, void *stream) {
    return launch_matvec("mvb_matvec", kQ8F32, gs, wq, ws, xq, xs, nullptr, out, n, d, kXQuantized,
                         static_cast<cudaStream_t>(stream));
}

extern "C" int mvb_qmatvec4(const void *w, const void *ws, const float *x, float *out, int n, int d, int wbits,
                            void *stream) {
    if (wbits != 4 && wbits != 8) {
        set_error("mvb_qmatvec4: unsupported wbits=%d (need 4 or 8)", wbits);
        return -1;
    }
    return launch_matvec("mvb_qmatvec4", wbits == 4 ? kQ4F16 : kQ8F16, 32, w, ws, nullptr, nullptr, x, out, n, d,
                         kXQuantizeQwen, static_cast<cudaStream_t>(stream));
}

extern "C" int mvb_qmatvec(const void *wq, const void *ws, const float *x, float *out, int n, int d, int gs,
                           void *stream) {
    return launch_matvec("mvb_qmatvec", kQ8F32, gs, wq, ws, nullptr, nullptr, x, out, n, d, kXQuantizeRunq,
                         static_cast<cudaStream_t>(stream));
}

