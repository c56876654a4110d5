// Host side of expf_ref.h: the table of inputs where the host C library's expf is not the correctly rounded
// value (or where the exact value sits within 2^-40 of a rounding midpoint), built by calling that expf on every
// float of [-104, 89] with all host threads, cached on disk, and uploaded as an open-addressing hash table.
//
// The cache lives in $MVB_CACHE_DIR, else $XDG_CACHE_HOME/mvb, else $HOME/.cache/mvb (made 0700), as a file made
// 0600; a cache file is used only if this user owns it, nobody else may write it, its length matches its entry
// count, every key lies in the table's domain and its checksum matches. Anything else is rebuilt.
#include <errno.h>
#include <fcntl.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "expf_ref.h"
#include "mvb_runtime.h"

namespace mvb {
namespace {

constexpr float kLo = -104.0f, kHi = 89.0f;
constexpr uint32_t kMagic = 0x32465845u;  // "EXF2": header, entries, then a checksum

struct Entry {
    uint32_t key, val;
};

struct HostTable {
    std::vector<Entry> entries;
    float max_delta = 0.0f;  // largest midpoint distance (ulps) of an input where the library is not correctly rounded
    bool ok = false;
};

std::mutex g_mu;
HostTable g_host;
std::map<unsigned long long, ExpTable> g_dev;  // the uploaded table of each CUDA context (by unique context ID)

uint32_t bits(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}

float from_bits(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}

// midpoint distance of d from the rounding midpoint on its side of c = (float)d, in ulps; the formula the device uses
double midpoint_delta(double d, float c) {
    const float nb = d >= (double)c ? nextafterf(c, INFINITY) : nextafterf(c, -INFINITY);
    const double gap = fabs((double)nb - (double)c);
    if (!(gap > 0.0)) return 1.0;
    return fabs(d - 0.5 * ((double)c + (double)nb)) / gap;
}

void scan(uint32_t first, uint32_t last, std::vector<Entry> *out, float *max_delta) {
    float md = 0.0f;
    for (uint64_t b = first; b <= last; b++) {
        const float x = from_bits((uint32_t)b);
        const float lib = expf(x);
        const double d = exp((double)x);
        const float c = (float)d;
        const bool differs = bits(lib) != bits(c);
        const bool near_mid = fabs(d - 0.5 * ((double)c + (double)(d >= (double)c ? nextafterf(c, INFINITY)
                                                                                    : nextafterf(c, -INFINITY)))) <=
                              fabs(d) * 0x1p-40;
        if (differs || near_mid) out->push_back(Entry{(uint32_t)b, bits(lib)});
        if (differs) md = std::max(md, (float)midpoint_delta(d, c));
    }
    *max_delta = md;
}

// A fingerprint of this host's expf and exp, so a cache from another library version is never used.
std::string fingerprint() {
    uint64_t h = 1469598103934665603ull;
    for (int i = 0; i < 4096; i++) {
        const float x = kLo + (kHi - kLo) * (float)i / 4096.0f;
        const uint32_t a = bits(expf(x)), b = bits((float)exp((double)x));
        h = (h ^ a) * 1099511628211ull;
        h = (h ^ b) * 1099511628211ull;
    }
    char s[32];
    snprintf(s, sizeof s, "%016llx", (unsigned long long)h);
    return s;
}

// The cache directory (created 0700 where it is this library's own), or "" if there is none.
std::string cache_dir() {
    const char *d = getenv("MVB_CACHE_DIR");
    if (d && *d) return d;
    std::string base;
    if ((d = getenv("XDG_CACHE_HOME")) && *d) base = d;
    else if ((d = getenv("HOME")) && *d) base = std::string(d) + "/.cache";
    else return "";
    mkdir(base.c_str(), 0700);  // may exist already
    const std::string dir = base + "/mvb";
    if (mkdir(dir.c_str(), 0700) != 0 && errno != EEXIST) return "";
    return dir;
}

std::string cache_path() {
    const std::string dir = cache_dir();
    return dir.empty() ? "" : dir + "/expf_v2_" + fingerprint() + ".bin";
}

uint64_t checksum(const HostTable &t) {
    uint64_t h = 1469598103934665603ull;
    auto mix = [&](uint32_t v) { h = (h ^ v) * 1099511628211ull; };
    mix(bits(t.max_delta));
    for (const Entry &e : t.entries) {
        mix(e.key);
        mix(e.val);
    }
    return h;
}

// A key of the table's domain: the bits of a float in [-104, -0] or [+0, 89].
bool in_domain(uint32_t key) {
    return (key >= bits(-0.0f) && key <= bits(kLo)) || key <= bits(kHi);
}

bool load_cache(HostTable *t) {
    const std::string path = cache_path();
    if (path.empty()) return false;
    const int fd = open(path.c_str(), O_RDONLY | O_NOFOLLOW);
    if (fd < 0) return false;
    struct stat st;
    FILE *f = fstat(fd, &st) == 0 ? fdopen(fd, "rb") : nullptr;
    if (!f) {
        close(fd);
        return false;
    }
    uint32_t hdr[2];
    float md;
    uint64_t sum = 0;
    // owned by this user, writable by nobody else, a regular file whose length matches its entry count
    bool ok = S_ISREG(st.st_mode) && st.st_uid == geteuid() && !(st.st_mode & 022) && fread(hdr, 4, 2, f) == 2 &&
              hdr[0] == kMagic && fread(&md, 4, 1, f) == 1 && md >= 0.0f && md <= 1.0f &&
              (uint64_t)st.st_size == 12 + (uint64_t)hdr[1] * sizeof(Entry) + 8 && hdr[1] < (1u << 24);
    if (ok) {
        t->entries.resize(hdr[1]);
        t->max_delta = md;
        ok = fread(t->entries.data(), sizeof(Entry), hdr[1], f) == hdr[1] && fread(&sum, 8, 1, f) == 1 &&
             sum == checksum(*t);
        for (size_t i = 0; ok && i < t->entries.size(); i++) ok = in_domain(t->entries[i].key);
    }
    fclose(f);
    if (!ok) {
        t->entries.clear();
        t->max_delta = 0.0f;
    }
    return ok;
}

void save_cache(const HostTable &t) {
    const std::string path = cache_path();
    if (path.empty()) return;
    const std::string tmp = path + ".tmp" + std::to_string((long)getpid());
    const int fd = open(tmp.c_str(), O_WRONLY | O_CREAT | O_EXCL | O_NOFOLLOW, 0600);
    if (fd < 0) return;
    FILE *f = fdopen(fd, "wb");
    if (!f) {
        close(fd);
        remove(tmp.c_str());
        return;
    }
    const uint32_t hdr[2] = {kMagic, (uint32_t)t.entries.size()};
    const uint64_t sum = checksum(t);
    bool ok = fwrite(hdr, 4, 2, f) == 2 && fwrite(&t.max_delta, 4, 1, f) == 1 &&
              fwrite(t.entries.data(), sizeof(Entry), t.entries.size(), f) == t.entries.size() &&
              fwrite(&sum, 8, 1, f) == 1;
    ok = fclose(f) == 0 && ok;
    if (ok) rename(tmp.c_str(), path.c_str());
    else remove(tmp.c_str());
}

void build_host() {
    if (g_host.ok) return;
    if (load_cache(&g_host)) {
        g_host.ok = true;
        return;
    }
    // negative inputs -0 .. -104 and positive inputs +0 .. 89, split over all host threads
    const uint32_t ranges[2][2] = {{bits(-0.0f), bits(kLo)}, {bits(0.0f), bits(kHi)}};
    unsigned nt = std::thread::hardware_concurrency();
    nt = nt ? std::min(nt, 256u) : 4;
    std::vector<std::vector<Entry>> parts(2 * nt);
    std::vector<float> md(2 * nt, 0.0f);
    std::vector<std::thread> th;
    for (int r = 0; r < 2; r++) {
        const uint64_t a = ranges[r][0], b = ranges[r][1], n = b - a + 1;
        for (unsigned i = 0; i < nt; i++) {
            const uint64_t lo = a + n * i / nt, hi = a + n * (i + 1) / nt - 1;
            if (lo > hi) continue;
            th.emplace_back(scan, (uint32_t)lo, (uint32_t)hi, &parts[r * nt + i], &md[r * nt + i]);
        }
    }
    for (auto &t : th) t.join();
    for (unsigned i = 0; i < 2 * nt; i++) {
        g_host.entries.insert(g_host.entries.end(), parts[i].begin(), parts[i].end());
        g_host.max_delta = std::max(g_host.max_delta, md[i]);
    }
    g_host.ok = true;
    save_cache(g_host);
}

}  // namespace

ExpTable expf_table_device() {
    std::lock_guard<std::mutex> lock(g_mu);
    ExpTable t = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return t;
    // a table uploaded in an earlier context of this device (before a cudaDeviceReset) is gone: key by context
    const unsigned long long ctx = current_context_id();
    auto it = ctx ? g_dev.find(ctx) : g_dev.end();
    if (it != g_dev.end()) return it->second;
    build_host();
    uint32_t slots = 1;
    while (slots < 4 * g_host.entries.size() + 16) slots <<= 1;
    std::vector<uint64_t> h(slots, (uint64_t)kExpEmpty);
    uint32_t max_probe = 0;
    for (const Entry &e : g_host.entries) {
        uint32_t p = exp_hash(e.key) & (slots - 1), n = 0;
        while ((uint32_t)h[p] != kExpEmpty) {
            p = (p + 1) & (slots - 1);
            n++;
        }
        h[p] = ((uint64_t)e.val << 32) | e.key;
        max_probe = std::max(max_probe, n);
    }
    uint64_t *d = nullptr;
    cudaError_t err = cudaMalloc(&d, (size_t)slots * 8);
    if (err == cudaSuccess) err = cudaMemcpy(d, h.data(), (size_t)slots * 8, cudaMemcpyHostToDevice);
    if (err != cudaSuccess) {
        set_error("expf table upload failed: %s", cudaGetErrorString(err));
        if (d) cudaFree(d);
        return t;
    }
    t.slots = d;
    t.mask = slots - 1;
    t.max_probe = max_probe;
    // probe whenever an input could be one of the recorded misroundings: their largest measured midpoint
    // distance plus a margin for the few-double-ulp difference between host and device exp; if the library ever
    // misrounded far from a midpoint, probe always
    t.thresh = g_host.max_delta < 0.25f ? g_host.max_delta + 1e-4f : 1.0f;
    t.lo = kLo;
    t.hi = kHi;
    const unsigned long long ctx_now = current_context_id();  // the upload made the context current if needed
    if (ctx_now) g_dev[ctx_now] = t;
    return t;
}

__global__ void expf_eval_kernel(const float *x, float *y, int n, const ExpTable t) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = expf_ref(x[i], t);
}

}  // namespace mvb

// Evaluates the device expf on n inputs (device pointers) and reports the table size and probe threshold, so
// tests can compare it with the host library's expf. 0, or -1.
extern "C" int mvb_expf_eval(const float *x, float *y, int n, int *entries, float *thresh, void *stream) {
    const mvb::ExpTable t = mvb::expf_table_device();
    if (!t.slots) return -1;
    if (entries) *entries = (int)mvb::g_host.entries.size();
    if (thresh) *thresh = t.thresh;
    if (n > 0) {
        mvb::expf_eval_kernel<<<(n + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, y, n, t);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) {
            mvb::set_error("mvb_expf_eval: %s", cudaGetErrorString(e));
            return -1;
        }
    }
    return 0;
}
