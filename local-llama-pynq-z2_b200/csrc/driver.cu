// The reference's board-driver C ABI (driver/matvec_fpga.h) served by a B200. See include/matvec_fpga.h for
// the contract. Replaces driver/matvec_fpga.cpp:
//   XRT/zocl CMA buffers (fpga_alloc_try, cpp:126-148)          -> pinned host buffer + HBM twin; "phys" = the
//                                                                 twin's device address
//   AXI-Lite register writes + ap_start (fpga_matvec, cpp:173-199; fpga_matvec4, cpp:207-233)
//                                                               -> argument validation, host<->HBM copies, launch
//   ap_done busy poll with TIMEOUT_S (run_kernel, cpp:157-171)  -> poll of a mapped completion word against a
//                                                                 deadline
// State is process-global and not thread-safe, like the reference's static globals (cpp:50-56).
//
// A call is one kernel launch: xq/xs are read from the caller's pinned buffer on the host and travel inside the
// launch's parameters (no upload copy), the kernel's last CTA copies the result rows into the caller's pinned buffer,
// which the device addresses directly (no download copy), then writes the call's number into a completion word in
// mapped host memory, and the call returns once the host sees that number there (the stream is asked about errors
// every 1024 polls).
//
// MATVEC_STATS=1 (environment, read by fpga_open) times every call: host time to enqueue, device time of the kernel
// (CUDA events), and the wait for completion; fpga_close() prints the means over the calls that uploaded no weights
// as one "matvec stats: {...}" JSON line on stderr.
#include <errno.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include <atomic>
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
    char *hdev;      // the pinned host memory as the device addresses it (kernels read and write it directly)
};

struct Stats {
    cudaEvent_t ev[4] = {};  // before the activation upload, before the launch, after the kernel, after the download
    double calls = 0, enqueue_us = 0, h2d_us = 0, kernel_us = 0, d2h_us = 0, wait_us = 0, total_us = 0;
    double upload_calls = 0;  // calls that also uploaded weights (first use), left out of the means
    double between_us = 0;    // host time from the return of the previous call to the entry of this one
    double t_return = 0;      // when the previous call returned (0: none yet)
};

struct Driver {
    bool open = false;
    bool failed = false;                     // a call timed out: its copies may still land, so refuse further calls
    int device = 0;
    cudaStream_t stream = nullptr;
    std::map<uint64_t, Buffer> bufs;         // keyed by device base address
    std::map<uint64_t, uint64_t> resident;   // weight byte ranges [first, second) already uploaded (merged)
    // weight ranges whose device address is not 16-byte aligned (fpga_matvec accepts any int8 address, as the
    // reference does): an aligned device copy per range, made on first use, keyed by (address, length)
    std::map<std::pair<uint64_t, size_t>, void *> shadows;
    unsigned *last = nullptr;                // the call kernel's last-CTA counter (device, back to 0 after every call)
    // the call's completion word: pinned host memory the kernel's last CTA writes the call's number into
    volatile unsigned *flag = nullptr;
    unsigned *flag_dev = nullptr;
    unsigned seq = 0;
    size_t total = 0;
    size_t limit = 0;                        // MATVEC_ALLOC_LIMIT, 0 = none
    double timeout_s = 5.0;                  // MATVEC_TIMEOUT_S, reference TIMEOUT_S (cpp:34)
    char last_alloc_err[256] = "";
    bool stats_on = false;                   // MATVEC_STATS
    Stats stats;
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
// *uploaded is set when this call copied anything.
bool ensure_resident(const Buffer &b, uint64_t addr, size_t len, bool *uploaded) {
    const uint64_t end = addr + len;
    auto it = drv.resident.upper_bound(addr);
    if (it != drv.resident.begin()) {
        auto prev = std::prev(it);
        if (prev->first <= addr && prev->second >= end) return true;
    }
    *uploaded = true;
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
int wait_done(const char *who, unsigned seq, int n, int d, int arg, const char *argname) {
    // The kernel's last CTA writes seq into the mapped completion word after the output (a system-scope fence
    // between them): polling that word sees the end of the call sooner than an event would. Every 1024 polls the
    // stream is asked about errors and the deadline is checked.
    const double deadline = now_s() + drv.timeout_s;
    for (unsigned i = 1;; i++) {
        if (*drv.flag == seq) {
            std::atomic_thread_fence(std::memory_order_acquire);  // the output is read after the word
            return 0;
        }
#if defined(__x86_64__) || defined(__i386__)
        __builtin_ia32_pause();  // a polite spin: the core's other hardware thread keeps its issue slots
#endif
        if (i % 1024 == 0) {
            const cudaError_t e = cudaStreamQuery(drv.stream);
            if (e != cudaSuccess && e != cudaErrorNotReady) {
                set_error("%s: device error: %s (n=%d d=%d %s=%d)", who, cudaGetErrorString(e), n, d, argname, arg);
                return -1;
            }
            if (e == cudaSuccess && *drv.flag != seq) {
                set_error("%s: the kernel ended without signalling completion (n=%d d=%d %s=%d)", who, n, d, argname,
                          arg);
                return -1;
            }
            if (now_s() > deadline) {
                set_error("%s: kernel did not finish in %g s (n=%d d=%d %s=%d)", who, drv.timeout_s, n, d, argname,
                          arg);
                drv.failed = true;  // its output copy may still land: no later call may reuse the buffers
                return -1;
            }
        }
    }
}

// An aligned device copy of the weight range [addr, addr + len) of buffer b (whose device address is misaligned),
// made on first use; null on failure.
void *shadow_of(const Buffer &b, uint64_t addr, size_t len, bool *uploaded) {
    const auto key = std::make_pair(addr, len);
    auto it = drv.shadows.find(key);
    if (it != drv.shadows.end()) return it->second;
    void *p = nullptr;
    if (cudaMalloc(&p, len) != cudaSuccess) return nullptr;
    if (cudaMemcpyAsync(p, b.host + (addr - b.dev), len, cudaMemcpyHostToDevice, drv.stream) != cudaSuccess) {
        cudaFree(p);
        return nullptr;
    }
    *uploaded = true;
    drv.shadows[key] = p;
    return p;
}

// One synchronous matvec through host buffers: weights resident, activations up, result down.
int run_call(const char *who, int fmt, int gs, uint64_t w, uint64_t ws, uint64_t xq, uint64_t xs, uint64_t out,
             int n, int d, int arg, const char *argname) {
    if (drv.failed) {
        set_error("%s: an earlier call timed out and its copies may still be in flight; call fpga_close()", who);
        return -1;
    }
    const double t_entry = drv.stats_on ? now_s() : 0.0;
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
    bool uploaded = false;
    const void *wdev = (const void *)w;
    if (w & 15) {  // a misaligned int8 plane (fpga_matvec only; fpga_matvec4 requires 64-byte alignment)
        wdev = shadow_of(*bw, w, wbytes, &uploaded);
        if (!wdev) {
            set_error("%s: cannot make an aligned copy of the weights at a misaligned address", who);
            return -1;
        }
    } else if (!ensure_resident(*bw, w, wbytes, &uploaded)) {
        set_error("%s: weight upload failed: %s", who, cudaGetErrorString(cudaGetLastError()));
        return -1;
    }
    if (!ensure_resident(*bs, ws, sbytes, &uploaded)) {
        set_error("%s: weight upload failed: %s", who, cudaGetErrorString(cudaGetLastError()));
        return -1;
    }
    if (drv.stats_on) cudaEventRecord(drv.stats.ev[0], drv.stream);
    if (drv.stats_on) cudaEventRecord(drv.stats.ev[1], drv.stream);
    int rc = launch_matvec_call(who, fmt, gs, wdev, (const void *)ws,
                                reinterpret_cast<const int8_t *>(bq->host + (xq - bq->dev)),
                                reinterpret_cast<const float *>(bx->host + (xs - bx->dev)), (float *)out,
                                reinterpret_cast<float *>(bo->hdev + (out - bo->dev)), drv.last, drv.flag_dev,
                                ++drv.seq, n, d, drv.stream);
    if (rc) return -1;
    if (drv.stats_on) {
        cudaEventRecord(drv.stats.ev[2], drv.stream);
        cudaEventRecord(drv.stats.ev[3], drv.stream);
    }
    const double t_enq = drv.stats_on ? now_s() : 0.0;
    rc = wait_done(who, drv.seq, n, d, arg, argname);
    if (rc == 0 && drv.stats_on) {
        Stats &st = drv.stats;
        if (uploaded) {
            st.upload_calls++;
        } else {
            const double t_done = now_s();
            float ms[3] = {0, 0, 0};
            for (int i = 0; i < 3; i++) cudaEventElapsedTime(&ms[i], st.ev[i], st.ev[i + 1]);
            st.calls++;
            if (st.t_return > 0) st.between_us += (t_entry - st.t_return) * 1e6;
            st.enqueue_us += (t_enq - t_entry) * 1e6;
            st.wait_us += (t_done - t_enq) * 1e6;
            st.total_us += (t_done - t_entry) * 1e6;
            st.h2d_us += ms[0] * 1e3;
            st.kernel_us += ms[1] * 1e3;
            st.d2h_us += ms[2] * 1e3;
        }
        st.t_return = now_s();
    }
    return rc;
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
    if (const char *e = getenv("FPGA_MEMIDX")) {  // reference: memory bank index (cpp:83-91)
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
    double limit = 0, timeout = 5.0, stats = 0;
    if (!env_number("MATVEC_ALLOC_LIMIT", &limit) || !env_number("MATVEC_TIMEOUT_S", &timeout) || timeout <= 0 ||
        !env_number("MATVEC_STATS", &stats)) {
        set_error("fpga: bad MATVEC_ALLOC_LIMIT, MATVEC_TIMEOUT_S or MATVEC_STATS");
        return -1;
    }
    if ((err = cudaSetDevice(dev)) != cudaSuccess ||
        (err = cudaStreamCreateWithFlags(&drv.stream, cudaStreamNonBlocking)) != cudaSuccess ||
        (err = cudaMalloc(&drv.last, sizeof(unsigned))) != cudaSuccess ||
        (err = cudaMemset(drv.last, 0, sizeof(unsigned))) != cudaSuccess ||
        (err = cudaHostAlloc((void **)&drv.flag, sizeof(unsigned), cudaHostAllocPortable | cudaHostAllocMapped)) !=
            cudaSuccess ||
        (err = cudaHostGetDevicePointer((void **)&drv.flag_dev, (void *)drv.flag, 0)) != cudaSuccess) {
        set_error("fpga: cannot open CUDA device %d: %s", dev, cudaGetErrorString(err));
        fpga_close();
        return -1;
    }
    *drv.flag = 0;
    drv.seq = 0;
    drv.stats_on = stats != 0;
    drv.stats = Stats{};
    for (int i = 0; drv.stats_on && i < 4; i++)
        if ((err = cudaEventCreate(&drv.stats.ev[i])) != cudaSuccess) {
            set_error("fpga: cannot create timing events: %s", cudaGetErrorString(err));
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
    void *h = nullptr, *d = nullptr, *hd = nullptr;
    cudaError_t e = cudaHostAlloc(&h, bytes, cudaHostAllocPortable | cudaHostAllocMapped);
    if (e == cudaSuccess) e = cudaHostGetDevicePointer(&hd, h, 0);
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
    drv.bufs[(uint64_t)d] = Buffer{(char *)h, (uint64_t)d, bytes, (char *)hd};
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
    if ((gs != 32 && gs != 64) || n <= 0 || n > kMaxN || n % gs || d <= 0) {  // reference checks (cpp:178-182)
        set_error("fpga_matvec: unsupported n=%d d=%d gs=%d (need gs 32 or 64, n %% gs == 0, n <= %d)", n, d, gs,
                  kMaxN);
        return -1;
    }
    // The reference checks no alignment (cpp:178); neither is wq/xq's needed here (a misaligned int8 plane or
    // vector is read from an aligned device copy). The fp32 arrays ws/xs/out must sit on 4 bytes, as the host's own
    // float pointers at the same offsets must for C.
    if ((ws | xs | out) & 3) {
        set_error("fpga_matvec: ws/xs/out must be 4-byte aligned (fp32 arrays)");
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
    // the reference's checks (cpp:212-216)
    if ((wbits != 4 && wbits != 8) || n <= 0 || n > kMaxN || n % 32 || d <= 0 || ((w | ws | xq | xs | out) & 63)) {
        set_error("fpga_matvec4: unsupported n=%d d=%d wbits=%d or a buffer not 64-byte aligned "
                  "(need wbits 4 or 8, n %% 32 == 0, n <= %d)", n, d, wbits, kMaxN);
        return -1;
    }
    return run_call("fpga_matvec4", wbits == 4 ? kQ4F16 : kQ8F16, 32, w, ws, xq, xs, out, n, d, wbits, "wbits");
}

extern "C" void fpga_close(void) {
    if (drv.stream) cudaStreamSynchronize(drv.stream);
    if (drv.stats_on) {
        const Stats &st = drv.stats;
        const double c = st.calls > 0 ? st.calls : 1;
        fprintf(stderr,
                "matvec stats: {\"calls\": %.0f, \"us_per_call\": %.2f, \"host_enqueue_us\": %.2f, "
                "\"upload_us\": %.2f, \"kernel_us\": %.2f, \"event_us\": %.2f, \"completion_wait_us\": %.2f, "
                "\"host_between_calls_us\": %.2f, \"calls_with_weight_upload\": %.0f}\n",
                st.calls, st.total_us / c, st.enqueue_us / c, st.h2d_us / c, st.kernel_us / c, st.d2h_us / c,
                st.wait_us / c, st.between_us / c, st.upload_calls);
        for (cudaEvent_t e : st.ev)
            if (e) cudaEventDestroy(e);
        drv.stats = Stats{};
        drv.stats_on = false;
    }
    for (auto &kv : drv.bufs) {
        cudaFreeHost(kv.second.host);
        cudaFree((void *)kv.second.dev);
    }
    for (auto &kv : drv.shadows) cudaFree(kv.second);
    drv.shadows.clear();
    if (drv.last) cudaFree(drv.last);
    drv.last = nullptr;
    drv.bufs.clear();
    drv.resident.clear();
    if (drv.flag) cudaFreeHost((void *)drv.flag);
    drv.flag = nullptr;
    drv.flag_dev = nullptr;
    drv.seq = 0;
    if (drv.stream) cudaStreamDestroy(drv.stream);
    drv.stream = nullptr;
    drv.total = 0;
    drv.failed = false;
    drv.open = false;
}
