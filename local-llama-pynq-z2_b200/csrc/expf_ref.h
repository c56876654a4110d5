// expf with the host C library's exact results, on the device.
//
// The reference's SiLU and softmax call the C library's expf (qwen.c:350, :560). glibc's expf is not correctly
// rounded: on about 8e-5 of the float inputs in [-104, 89] it returns the neighbour of the correctly rounded
// value. Because every matvec input is re-quantized to int8, a one-ulp difference in one activation can flip a
// rounding and grow through the layers, so the decode must reproduce those results exactly.
//
// How: the device computes the correctly rounded value from a double-precision exp. At load time the host calls
// its own expf on every float of the domain and records, in a hash table, each input where the library's result
// differs from the correctly rounded one, plus every input whose exact result lies within 2^-40 (relative) of a
// float rounding midpoint (there a host/device difference of a few double ulps could round either way). A
// library result can only differ from the correctly rounded one when the exact value is close to a midpoint;
// the build measures how close every recorded input is and the device probes the table only when its value is
// that close (about 0.4% of calls). The table is built once per machine and cached on disk.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace mvb {

struct ExpTable {
    const uint64_t *slots;  // (result bits << 32) | input bits; empty slots hold kExpEmpty in the low word
    uint32_t mask;          // slots - 1 (power of two)
    uint32_t max_probe;     // longest probe sequence of any key
    float thresh;           // probe when |exp(x) - nearest midpoint| <= thresh * ulp
    float lo, hi;           // table domain
};

constexpr uint32_t kExpEmpty = 0xFFFFFFFFu;

__host__ __device__ inline uint32_t exp_hash(uint32_t k) {
    k ^= k >> 16;
    k *= 0x7feb352dU;
    k ^= k >> 15;
    k *= 0x846ca68bU;
    k ^= k >> 16;
    return k;
}

#ifdef __CUDACC__
// The host C library's expf(x), given a table built by expf_table_device().
__device__ __forceinline__ float expf_ref(float x, const ExpTable t) {
    const double d = exp((double)x);
    const float c = (float)d;
    if (!(x >= t.lo && x <= t.hi) || !t.slots) return c;
    // distance of d from the midpoint between c and its neighbour on d's side, in ulps of that interval
    const float nb = d >= (double)c ? nextafterf(c, INFINITY) : nextafterf(c, -INFINITY);
    const double gap = fabs((double)nb - (double)c);
    if (!(gap > 0.0)) return c;
    const double delta = fabs(d - 0.5 * ((double)c + (double)nb)) / gap;
    if (delta > (double)t.thresh) return c;
    const uint32_t key = __float_as_uint(x);
    uint32_t h = exp_hash(key) & t.mask;
    for (uint32_t i = 0; i <= t.max_probe; i++) {
        const uint64_t e = __ldg(reinterpret_cast<const unsigned long long *>(t.slots + h));
        const uint32_t k = (uint32_t)e;
        if (k == key) return __uint_as_float((uint32_t)(e >> 32));
        if (k == kExpEmpty) break;
        h = (h + 1) & t.mask;
    }
    return c;
}
#endif

// Builds (or loads from the cache) the table for the current device and returns it; slots stay allocated for
// the life of the process. On failure returns a table with slots == nullptr (expf_ref then returns the
// correctly rounded value) and sets the library error.
ExpTable expf_table_device();

}  // namespace mvb
