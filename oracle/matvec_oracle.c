/* CPU restatement of the reference's group-quantized matvec path. TEST INFRASTRUCTURE ONLY.
 *
 * Only the tests, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load this file's library, and
 * only as the checker. The product (libmatvec_b200.so) never calls it and has no CPU fallback.
 *
 * Parity pin: every function here is checked bit-for-bit against the reference's own C (qwen/qwen.c and
 * runq/runq.c, compiled unchanged into oracle/_ref/ by oracle/Makefile) on the committed fixtures in
 * tests/golden/ (made by tests/golden/make_golden.py).
 *
 * Arithmetic follows the reference exactly: int32 sums inside a group, then per group
 * p = ((float)isum * wscale) * xscale in two separate fp32 multiplies (no FMA), and the p of a row added
 * in group order into a float that starts at 0. Build with -ffp-contract=off.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

/* fp16 bits -> fp32, as qwen/qwen.c:84-94 does it: exact for zero, subnormals and normals. The reference
 * treats exponent field 31 like any other exponent (its scales hold no inf/nan), so 31 maps to the finite
 * value 2^16 * (1 + m/1024), not to inf/nan. */
float orc_f16(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t e = (h >> 10) & 31u, m = h & 1023u;
    uint32_t bits;
    if (e == 0 && m == 0) {
        bits = sign;
    } else if (e == 0) {
        /* subnormal: m * 2^-24; shift the leading one into the implicit bit */
        int shift = 0;
        while (!(m & 1024u)) { m <<= 1; shift++; }
        m &= 1023u;
        bits = sign | ((uint32_t)(113 - shift) << 23) | (m << 13);
    } else {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* float -> int8_t as the reference's casts behave on x86-64 (qwen.c:362, runq.c:266): through a 32-bit
 * conversion that turns NaN and values outside int32 into INT32_MIN (low byte 0), then truncation to 8 bits.
 * C leaves such casts undefined; this is what gcc's cvttss2si/cvttsd2si produce, and it matters for groups whose
 * scale is subnormal (1/scale overflows to inf in qwen.c) or zero (0/0 in runq.c). */
static inline int8_t to_int8_x86(float r) {
    if (!(fabsf(r) < 2147483648.0f)) return 0;
    return (int8_t)(int32_t)r;
}

/* Activation quantization of qwen/qwen.c:355-364 (group size 32): scale = max|x| * (1/127),
 * inv = 1/scale (0 when scale is 0), q = roundf(x * inv), halves away from zero. */
void orc_quantize_qwen(int8_t *q, float *s, const float *x, int n) {
    for (int g = 0; g < n / 32; g++) {
        float amax = 0.0f;
        for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(x[32 * g + i]));
        float scale = amax * (1.0f / 127.0f);
        float inv = scale > 0.0f ? 1.0f / scale : 0.0f;
        s[g] = scale;
        for (int i = 0; i < 32; i++) q[32 * g + i] = to_int8_x86(roundf(x[32 * g + i] * inv));
    }
}

/* Activation quantization of runq/runq.c:244-270: scale = max|x| / 127, q = round(x / scale).
 * The reference divides by the scale (no reciprocal) and has no zero guard: an all-zero group divides
 * 0 by 0, and that NaN converts to 0 (to_int8_x86). */
void orc_quantize_runq(int8_t *q, float *s, const float *x, int n, int gs) {
    for (int g = 0; g < n / gs; g++) {
        float amax = 0.0f;
        for (int i = 0; i < gs; i++) {
            float a = fabsf(x[gs * g + i]);
            if (a > amax) amax = a;
        }
        float scale = amax / 127.0f;
        s[g] = scale;
        for (int i = 0; i < gs; i++) {
            q[gs * g + i] = to_int8_x86(roundf(x[gs * g + i] / scale));
        }
    }
}

/* Signed value of element k of a packed row: 4-bit planes keep element 2i in the low nibble of byte i and
 * 2i+1 in the high nibble, two's complement (qwen/qwen.c:445-448; tools/gguf2qwb.py:13-14). */
static inline int weight_at(const uint8_t *row, int k, int bits) {
    if (bits == 8) return (int8_t)row[k];
    int nib = (row[k >> 1] >> ((k & 1) * 4)) & 15;
    return nib >= 8 ? nib - 16 : nib;
}

/* Integer sum of group g of row i: sum over k < gs of w[i, g*gs + k] * xq[g*gs + k]. */
static inline int32_t group_sum(const uint8_t *row, const int8_t *xq, int g, int gs, int bits) {
    int32_t acc = 0;
    for (int k = 0; k < gs; k++) acc += weight_at(row, g * gs + k, bits) * (int32_t)xq[g * gs + k];
    return acc;
}

/* Per-group int32 sums of W (d x n) against xq: isum[i * (n/gs) + g]. */
void orc_group_sums(int32_t *isum, const uint8_t *w, const int8_t *xq, int n, int d, int gs, int bits) {
    const int ng = n / gs;
    const size_t row_bytes = (size_t)n * bits / 8;
    for (int i = 0; i < d; i++)
        for (int g = 0; g < ng; g++) isum[(size_t)i * ng + g] = group_sum(w + (size_t)i * row_bytes, xq, g, gs, bits);
}

/* matvec4 with fp16 weight scales (qwen/qwen.c:436-456, contract hls4/matvec4.h:1-21), wbits 4 or 8,
 * group size 32: out[i] = sum_g ((float)isum * f16(ws[i*ng + g])) * xs[g], groups in order. */
void orc_matvec_f16(float *out, const uint8_t *w, const uint16_t *ws, const int8_t *xq, const float *xs, int n, int d,
                    int bits) {
    const int ng = n / 32;
    const size_t row_bytes = (size_t)n * bits / 8;
    for (int i = 0; i < d; i++) {
        const uint8_t *row = w + (size_t)i * row_bytes;
        float val = 0.0f;
        for (int g = 0; g < ng; g++) {
            float p = (float)group_sum(row, xq, g, 32, bits) * orc_f16(ws[(size_t)i * ng + g]);
            p = p * xs[g];
            val = val + p;
        }
        out[i] = val;
    }
}

/* runq matvec with fp32 weight scales and group size 32 or 64 (runq/runq.c:430-458, contract hls/matvec.h:1-19):
 * out[i] = sum_g ((float)isum * ws[(i*n + g*gs)/gs]) * xs[g], groups in order. */
void orc_matvec_f32(float *out, const int8_t *wq, const float *ws, const int8_t *xq, const float *xs, int n, int d,
                    int gs) {
    const int ng = n / gs;
    for (int i = 0; i < d; i++) {
        const uint8_t *row = (const uint8_t *)wq + (size_t)i * n;
        float val = 0.0f;
        for (int g = 0; g < ng; g++) {
            float p = (float)group_sum(row, xq, g, gs, 8) * ws[(size_t)i * ng + g];
            p = p * xs[g];
            val = val + p;
        }
        out[i] = val;
    }
}

/* The host C library's expf over an array: the function qwen.c's softmax and SiLU call (qwen.c:350, :560). */
void orc_expf_array(const float *x, float *y, long n) {
    for (long i = 0; i < n; i++) y[i] = expf(x[i]);
}
