// Launchers of the matvec kernels and the device-pointer entry points of include/matvec_b200.h.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <map>
#include <mutex>

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

// Rows per CTA: enough tiles for ~4 CTAs per SM on 148 SMs, at most 32 rows so the in-order fold stays one
// warp and the product buffer stays small.
int rows_per_tile(int n, int d) {
    (void)n;
    const int target_tiles = 148 * 4;
    const int rt = (d + target_tiles - 1) / target_tiles;
    return rt < 1 ? 1 : (rt > 32 ? 32 : rt);
}

template <int FMT, int GS>
static cudaError_t launch(MatvecParams p, cudaStream_t stream, bool pdl) {
    p.rt = rows_per_tile(p.n, p.d);
    const size_t smem = matvec_smem_bytes(p.n, GS, p.rt);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((p.d + p.rt - 1) / p.rt);
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
    return cudaLaunchKernelEx(&cfg, matvec_kernel<FMT, GS>, p);
}

static bool aligned(const void *p, uintptr_t a) { return ((uintptr_t)p & (a - 1)) == 0; }

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
    if (!quantized && !(xmode == kXQuantizeQwen || xmode == kXQuantizeRunq)) {
        set_error("%s: bad activation mode %d", who, xmode);
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
    if (fmt == kQ4F16) e = launch<kQ4F16, 32>(p, stream, pdl);
    else if (fmt == kQ8F16) e = launch<kQ8F16, 32>(p, stream, pdl);
    else if (gs == 32) e = launch<kQ8F32, 32>(p, stream, pdl);
    else e = launch<kQ8F32, 64>(p, stream, pdl);
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

