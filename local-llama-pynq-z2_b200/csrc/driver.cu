// The reference's board-driver C ABI (driver/matvec_fpga.h) served by a B200. See include/matvec_fpga.h for
// the contract. Replaces driver/matvec_fpga.cpp:
//   XRT/zocl CMA buffers (cpp:163-191)       -> pinned host buffer + HBM twin; "phys" = the twin's device address
//   AXI-Lite register writes + ap_start (cpp:210-269) -> argument validation, host<->HBM copies, kernel launch
//   ap_done busy poll with TIMEOUT_S (cpp:193-207)    -> cudaEventQuery poll against a deadline
// State is process-global and not thread-safe, like the reference's static globals (cpp:87-93).
#include <errno.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include <map>
#include <vector>

#include "../../include/matvec_b200.h"
#include "matvec_kernels.cuh"
#include "mvb_runtime.h"

using namespace mvb;

namespace {

struct Buffer {
    char *host;      // pinned host memory the caller writes and reads
    uint64_t dev;    // device twin (same size), what the caller passes as a "physical address"
    size_t size;
};

struct Driver {
    bool open = false;
    int device = 0;
    cudaStream_t stream = nullptr;
    cudaEvent_t done = nullptr;
    std::map<uint64_t, Buffer> bufs;         // keyed by device base address
    std::map<uint64_t, uint64_t> resident;   // weight byte ranges [first, second) already uploaded (merged)
    size_t total = 0;
    size_t limit = 0;                        // MATVEC_ALLOC_LIMIT, 0 = none
    double timeout_s = 5.0;                  // MATVEC_TIMEOUT_S, reference TIMEOUT_S (cpp:71)
    char last_alloc_err[256] = "";
};

Driver drv;

double now_s() {
    timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return t.tv_sec + t.tv_nsec * 1e-9;
}

// The buffer holding [addr, addr + len), or null.
Buffer *resolve(uint64_t addr, size_t len) {
    auto it = drv.bufs.upper_bound(addr);
    if (it == drv.bufs.begin()) return nullptr;
    --it;
    Buffer &b = it->second;
    if (addr < b.dev || addr - b.dev > b.size || len > b.size - (addr - b.dev)) return nullptr;
    return &b;
}

// Uploads [addr, addr + len) unless a previous call already did; weights are immutable after first use.
bool ensure_resident(const Buffer &b, uint64_t addr, size_t len) {
    const uint64_t end = addr + len;
    auto it = drv.resident.upper_bound(addr);
    if (it != drv.resident.begin()) {
        auto prev = std::prev(it);
        if (prev->first <= addr && prev->second >= end) return true;
    }
    cudaError_t e = cudaMemcpyAsync((void *)addr, b.host + (addr - b.dev), len, cudaMemcpyHostToDevice, drv.stream);
    if (e != cudaSuccess) return false;
    // insert [addr, end) and merge with overlapping or touching neighbours
    uint64_t lo = addr, hi = end;
    it = drv.resident.upper_bound(addr);
    if (it != drv.resident.begin()) {
        auto prev = std::prev(it);
        if (prev->second >= lo) {
            lo = prev->first;
            hi = std::max(hi, prev->second);
            drv.resident.erase(prev);
        }
    }
    it = drv.resident.lower_bound(lo);
    while (it != drv.resident.end() && it->first <= hi) {
        hi = std::max(hi, it->second);
        it = drv.resident.erase(it);
    }
    drv.resident[lo] = hi;
    return true;
}

// Waits for the stream's work with a deadline; 0, or -1 on timeout or a CUDA error.
int wait_done(const char *who, int n, int d, int arg, const char *argname) {
    cudaError_t e = cudaEventRecord(drv.done, drv.stream);
    if (e != cudaSuccess) {
        set_error("%s: %s", who, cudaGetErrorString(e));
        return -1;
    }
    const double deadline = now_s() + drv.timeout_s;
    for (unsigned i = 1;; i++) {
        e = cudaEventQuery(drv.done);
        if (e == cudaSuccess) return 0;
        if (e != cudaErrorNotReady) {
            set_error("%s: device error: %s (n=%d d=%d %s=%d)", who, cudaGetErrorString(e), n, d, argname, arg);
            return -1;
        }
        if (i % 256 == 0 && now_s() > deadline) {
            set_error("%s: kernel did not finish in %g s (n=%d d=%d %s=%d)", who, drv.timeout_s, n, d, argname, arg);
            return -1;
        }
    }
}

// One synchronous matvec through host buffers: weights resident, activations up, result down.
int run_call(const char *who, int fmt, int gs, uint64_t w, uint64_t ws, uint64_t xq, uint64_t xs, uint64_t out,
             int n, int d, int arg, const char *argname) {
    const int ng = n / gs;
    const size_t wbytes = (size_t)d * n * (fmt == kQ4F16 ? 4 : 8) / 8;
    const size_t sbytes = (size_t)d * ng * (fmt == kQ8F32 ? 4 : 2);
    Buffer *bw = resolve(w, wbytes), *bs = resolve(ws, sbytes), *bq = resolve(xq, n), *bx = resolve(xs, ng * 4),
           *bo = resolve(out, (size_t)d * 4);
    if (!bw || !bs || !bq || !bx || !bo) {
        set_error("%s: an address range is not inside a buffer from fpga_alloc() (%s%s%s%s%s)", who,
                  bw ? "" : "w ", bs ? "" : "ws ", bq ? "" : "xq ", bx ? "" : "xs ", bo ? "" : "out");
        return -1;
    }
    if (!ensure_resident(*bw, w, wbytes) || !ensure_resident(*bs, ws, sbytes)) {
        set_error("%s: weight upload failed: %s", who, cudaGetErrorString(cudaGetLastError()));
        return -1;
    }
    cudaError_t e;
    if (bq == bx && xs >= xq && xs - xq <= 65536) {  // one copy when the scales sit just after the values
        e = cudaMemcpyAsync((void *)xq, bq->host + (xq - bq->dev), xs + ng * 4 - xq, cudaMemcpyHostToDevice,
                            drv.stream);
    } else {
        e = cudaMemcpyAsync((void *)xq, bq->host + (xq - bq->dev), n, cudaMemcpyHostToDevice, drv.stream);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync((void *)xs, bx->host + (xs - bx->dev), ng * 4, cudaMemcpyHostToDevice, drv.stream);
    }
    if (e != cudaSuccess) {
        set_error("%s: activation upload failed: %s", who, cudaGetErrorString(e));
        return -1;
    }
    if (launch_matvec(who, fmt, gs, (const void *)w, (const void *)ws, (const void *)xq, (const void *)xs, nullptr,
                      (float *)out, n, d, kXQuantized, drv.stream) != 0)
        return -1;
    e = cudaMemcpyAsync(bo->host + (out - bo->dev), (const void *)out, (size_t)d * 4, cudaMemcpyDeviceToHost,
                        drv.stream);
    if (e != cudaSuccess) {
        set_error("%s: result download failed: %s", who, cudaGetErrorString(e));
        return -1;
    }
    return wait_done(who, n, d, arg, argname);
}

bool env_number(const char *name, double *out) {
    const char *e = getenv(name);
    if (!e) return true;
    char *end;
    errno = 0;
    double v = strtod(e, &end);
    if (!*e || *end || errno || v < 0) return false;
    *out = v;
    return true;
}

}  // namespace

extern "C" int fpga_open(void) {
    if (drv.open) return 0;
    int dev = 0;
    if (const char *e = getenv("FPGA_MEMIDX")) {  // reference: memory bank index (cpp:120-128)
        char *end;
        long v = strtol(e, &end, 0);
        if (!*e || *end || v < 0) {
            set_error("fpga: bad FPGA_MEMIDX '%s'", e);
            return -1;
        }
        dev = (int)v;
    }
    int count = 0;
    cudaError_t err = cudaGetDeviceCount(&count);
    if (err != cudaSuccess || dev >= count) {
        set_error("fpga: no CUDA device %d (%s)", dev, err != cudaSuccess ? cudaGetErrorString(err) : "out of range");
        return -1;
    }
    double limit = 0, timeout = 5.0;
    if (!env_number("MATVEC_ALLOC_LIMIT", &limit) || !env_number("MATVEC_TIMEOUT_S", &timeout) || timeout <= 0) {
        set_error("fpga: bad MATVEC_ALLOC_LIMIT or MATVEC_TIMEOUT_S");
        return -1;
    }
    if ((err = cudaSetDevice(dev)) != cudaSuccess ||
        (err = cudaStreamCreateWithFlags(&drv.stream, cudaStreamNonBlocking)) != cudaSuccess ||
        (err = cudaEventCreateWithFlags(&drv.done, cudaEventDisableTiming)) != cudaSuccess) {
        set_error("fpga: cannot open CUDA device %d: %s", dev, cudaGetErrorString(err));
        fpga_close();
        return -1;
    }
    drv.device = dev;
    drv.limit = (size_t)limit;
    drv.timeout_s = timeout;
    drv.open = true;
    return 0;
}

extern "C" void *fpga_alloc_try(size_t bytes, uint64_t *phys) {
    if (!drv.open || !bytes || !phys) {
        snprintf(drv.last_alloc_err, sizeof drv.last_alloc_err, "%s",
                 !drv.open ? "fpga_open() not called" : (!bytes ? "zero size" : "null phys"));
        return nullptr;
    }
    if (drv.limit && drv.total + bytes > drv.limit) {
        snprintf(drv.last_alloc_err, sizeof drv.last_alloc_err,
                 "%zu bytes failed after %.1f MiB already allocated (MATVEC_ALLOC_LIMIT %zu)", bytes,
                 drv.total / 1048576.0, drv.limit);
        return nullptr;
    }
    cudaSetDevice(drv.device);
    void *h = nullptr, *d = nullptr;
    cudaError_t e = cudaHostAlloc(&h, bytes, cudaHostAllocPortable);
    if (e == cudaSuccess) e = cudaMalloc(&d, bytes);
    if (e == cudaSuccess) e = cudaMemsetAsync(d, 0, bytes, drv.stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(drv.stream);
    if (e != cudaSuccess) {
        snprintf(drv.last_alloc_err, sizeof drv.last_alloc_err, "%zu bytes failed after %.1f MiB already allocated: %s",
                 bytes, drv.total / 1048576.0, cudaGetErrorString(e));
        if (h) cudaFreeHost(h);
        if (d) cudaFree(d);
        cudaGetLastError();
        return nullptr;
    }
    memset(h, 0, bytes);
    drv.bufs[(uint64_t)d] = Buffer{(char *)h, (uint64_t)d, bytes};
    drv.total += bytes;
    *phys = (uint64_t)d;
    return h;
}

extern "C" void *fpga_alloc(size_t bytes, uint64_t *phys) {
    void *p = fpga_alloc_try(bytes, phys);
    if (!p) set_error("fpga_alloc: %s", drv.last_alloc_err);
    return p;
}

extern "C" int fpga_matvec(uint64_t wq, uint64_t ws, uint64_t xq, uint64_t xs, uint64_t out, int n, int d, int gs) {
    if (!drv.open) {
        set_error("fpga_matvec: fpga_open() not called");
        return -1;
    }
    if ((gs != 32 && gs != 64) || n <= 0 || n > kMaxN || n % gs || d <= 0) {  // reference checks (cpp:215-219)
        set_error("fpga_matvec: unsupported n=%d d=%d gs=%d (need gs 32 or 64, n %% gs == 0, n <= %d)", n, d, gs,
                  kMaxN);
        return -1;
    }
    if ((wq | xq) & 15 || (ws | xs | out) & 3) {  // the reference's AXI bursts need no alignment; 128-bit loads do
        set_error("fpga_matvec: wq/xq must be 16-byte and ws/xs/out 4-byte aligned");
        return -1;
    }
    return run_call("fpga_matvec", kQ8F32, gs, wq, ws, xq, xs, out, n, d, gs, "gs");
}

extern "C" int fpga_matvec4(uint64_t w, uint64_t ws, uint64_t xq, uint64_t xs, uint64_t out, int n, int d,
                            int wbits) {
    if (!drv.open) {
        set_error("fpga_matvec4: fpga_open() not called");
        return -1;
    }
    if ((wbits != 4 && wbits != 8) || n <= 0 || n > kMaxN || n % 32 || d <= 0 || ((w | ws | xq | xs | out) & 63)) {
        set_error("fpga_matvec4: unsupported n=%d d=%d wbits=%d or a buffer not 64-byte aligned "
                  "(need wbits 4 or 8, n %% 32 == 0, n <= %d)", n, d, wbits, kMaxN);
        return -1;
    }
    return run_call("fpga_matvec4", wbits == 4 ? kQ4F16 : kQ8F16, 32, w, ws, xq, xs, out, n, d, wbits, "wbits");
}

extern "C" void fpga_close(void) {
    if (drv.stream) cudaStreamSynchronize(drv.stream);
    for (auto &kv : drv.bufs) {
        cudaFreeHost(kv.second.host);
        cudaFree((void *)kv.second.dev);
    }
    drv.bufs.clear();
    drv.resident.clear();
    if (drv.done) cudaEventDestroy(drv.done);
    if (drv.stream) cudaStreamDestroy(drv.stream);
    drv.done = nullptr;
    drv.stream = nullptr;
    drv.total = 0;
    drv.open = false;
}
