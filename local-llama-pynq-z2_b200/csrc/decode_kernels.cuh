// Kernels of the device-resident decode step (qwen_decode.cu). Every kernel:
//   1. loads what does not depend on the previous kernel (its weight tile, into registers) and lets the next
//      kernel launch (griddepcontrol.launch_dependents), so with programmatic dependent launch the next kernel's
//      weight fetch overlaps this one;
//   2. waits for the previous kernel (griddepcontrol.wait) and turns its fp32 output into this kernel's int8
//      input in every CTA at once (rmsnorm + quantize, or quantize), reading it with L2 loads;
//   3. computes. Two kernels also have a tail run by their last CTA to finish (an atomic counter that this CTA
//      resets for the next step): the last layer's down projection normalizes x once for the 2,048-CTA head,
//      and the head picks the next token.
// The arithmetic of every step is qwen.c's, operation by operation (see qwen_decode.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "expf_ref.h"
#include "matvec_kernels.cuh"

namespace mvb {
namespace qwen {

constexpr int kImEnd = 151645, kEndOfText = 151643;  // qwen.c:31-32

struct State {
    int token;       // token of the current position
    int pos;         // current position
    int n_prompt;    // prompt length; < 0: the host supplies every token (no prompt feeding, no sampling)
    int n_gen;       // tokens generated so far
    unsigned long long key;  // argmax of the head: (orderable logit << 32) | ~row
    int last_row;    // head row of the last argmax
    int pad;
};

__device__ __forceinline__ float4 ld_cg4(const float *p) { return __ldcg(reinterpret_cast<const float4 *>(p)); }

// ((0 + x0^2) + x1^2) + ... in order (qwen.c:339), by one thread from shared memory (n % 16 == 0, 16-byte aligned).
// The squares are off the dependency chain and the next 16 values are loaded before the current 16 are added, so
// the loop runs at the latency of one fp32 add per element.
__device__ __forceinline__ float sum_squares_inorder(const float *x, int n) {
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
    float s = 0.0f;
    float4 c[4] = {x4[0], x4[1], x4[2], x4[3]};
    for (int j = 0; j < n; j += 16) {
        float4 nx[4];
        const bool more = j + 16 < n;
        if (more) {
#pragma unroll
            for (int i = 0; i < 4; i++) nx[i] = x4[(j + 16) / 4 + i];
        }
        float q[16];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            q[4 * i] = __fmul_rn(c[i].x, c[i].x);
            q[4 * i + 1] = __fmul_rn(c[i].y, c[i].y);
            q[4 * i + 2] = __fmul_rn(c[i].z, c[i].z);
            q[4 * i + 3] = __fmul_rn(c[i].w, c[i].w);
        }
#pragma unroll
        for (int i = 0; i < 16; i++) s = __fadd_rn(s, q[i]);
        if (more) {
#pragma unroll
            for (int i = 0; i < 4; i++) c[i] = nx[i];
        }
    }
    return s;
}

// ((0 + a0) + a1) + ... over a[0 .. n-1] in order, one thread, shared memory (any n, 16-byte aligned a).
__device__ __forceinline__ float sum_inorder(const float *a, int n) {
    float s = 0.0f;
    int j = 0;
    const float4 *a4 = reinterpret_cast<const float4 *>(a);
    if (n >= 16) {
        float4 c[4] = {a4[0], a4[1], a4[2], a4[3]};
        for (; j + 16 <= n; j += 16) {
            float4 nx[4];
            const bool more = j + 32 <= n;
            if (more) {
#pragma unroll
                for (int i = 0; i < 4; i++) nx[i] = a4[(j + 16) / 4 + i];
            }
#pragma unroll
            for (int i = 0; i < 4; i++) {
                s = __fadd_rn(s, c[i].x);
                s = __fadd_rn(s, c[i].y);
                s = __fadd_rn(s, c[i].z);
                s = __fadd_rn(s, c[i].w);
            }
            if (more) {
#pragma unroll
                for (int i = 0; i < 4; i++) c[i] = nx[i];
            }
        }
    }
    for (; j < n; j++) s = __fadd_rn(s, a[j]);
    return s;
}

// One group of 32 values held in registers, quantized like qwen.c:355-364 (the operations of quantize_group's
// qwen mode): returns the scale, q receives the int8 values.
__device__ __forceinline__ float quantize32_qwen(const float (&v)[32], int8_t (&q)[32]) {
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(v[i]));
    const float scale = __fmul_rn(amax, 1.0f / 127.0f);
    const float inv = scale > 0.0f ? __fdiv_rn(1.0f, scale) : 0.0f;
#pragma unroll
    for (int i = 0; i < 32; i++) q[i] = to_int8_x86(roundf(__fmul_rn(v[i], inv)));
    return scale;
}

// Quantizes v[0 .. n-1] (shared memory) per group of 32 like qwen.c:355-364 into xq/xs (global); whole CTA.
__device__ __forceinline__ void quantize_to_global(const float *v, int n, int8_t *xq, float *xs) {
    for (int g = threadIdx.x; g < n / 32; g += blockDim.x) {
        int8_t q[32];
        xs[g] = quantize_group<32>(v, g, kXQuantizeQwen, q);
        uint32_t w[8];
#pragma unroll
        for (int j = 0; j < 8; j++)
            w[j] = (uint32_t)(uint8_t)q[4 * j] | (uint32_t)(uint8_t)q[4 * j + 1] << 8 |
                   (uint32_t)(uint8_t)q[4 * j + 2] << 16 | (uint32_t)(uint8_t)q[4 * j + 3] << 24;
        uint4 *dst = reinterpret_cast<uint4 *>(xq + 32 * g);
        dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
        dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
    }
}

// rmsnorm (qwen.c:337-344) of xv (shared memory, n floats) with weight w, then quantize into xq/xs; whole CTA.
// xb is n floats of shared scratch.
__device__ __forceinline__ void rmsnorm_quantize(const float *xv, float *xb, const float *w, float eps, int n,
                                                 int8_t *xq, float *xs) {
    __shared__ float s_inv;
    __syncthreads();
    if (threadIdx.x == 0) {
        float ss = sum_squares_inorder(xv, n);
        ss = __fdiv_rn(ss, (float)n);
        ss = __fadd_rn(ss, eps);
        s_inv = __fdiv_rn(1.0f, __fsqrt_rn(ss));
    }
    __syncthreads();
    const float s = s_inv;
    for (int j = threadIdx.x; j < n; j += blockDim.x) xb[j] = __fmul_rn(w[j], __fmul_rn(s, xv[j]));
    __syncthreads();
    quantize_to_global(xb, n, xq, xs);
}

// Once every CTA of the grid has called this (after its global writes), returns true in exactly one CTA: the
// last to arrive, which then sees all their writes. That CTA resets the counter for the next launch.
__device__ __forceinline__ bool last_cta(int *counter) {
    __shared__ int s_last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(counter, 1) == (int)(gridDim.x * gridDim.y) - 1;
    __syncthreads();
    if (!s_last) return false;
    __threadfence();
    if (threadIdx.x == 0) *counter = 0;
    return true;
}

// ---------------------------------------------------------------------------------------------------------------
// embedding row of the current token (qwen.c:498-501), exact in fp32; also clears the head's argmax key.
__global__ void embed_kernel(const int8_t *emb_q, const uint16_t *emb_s, float *x, int dim, State *st) {
    allow_consumer();
    wait_for_producer();
    const int tok = __ldcg(&st->token);
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i == 0) st->key = 0ull;
    if (i < dim) {
        const size_t r = (size_t)tok * dim;
        x[i] = __fmul_rn(__int2float_rn(emb_q[r + i]), scale_from_f16(emb_s[r / 32 + i / 32]));
    }
}

// ---------------------------------------------------------------------------------------------------------------
enum Epilogue : int {
    kEpiStore = 0,     // out[row] = v
    kEpiResidual = 1,  // out[row] += v                                              (qwen.c:551, :565)
    kEpiSwiGLU = 2,    // tile = rows of w1 then the same rows of w3; out[row] = silu(g) * u   (qwen.c:558-562)
    kEpiHead = 3,      // out[row] = v, plus the argmax key                           (qwen.c:571, 591-598)
};

enum Prologue : int {
    kProQuantized = 0,  // xq/xs given (int8 + scales)
    kProQuant = 1,      // quantize the fp32 vector src                            (qwen.c:549, :563)
    kProNorm = 2,       // rmsnorm src with norm_w, then quantize                  (qwen.c:516-517, :554-555)
};

enum Tail : int {
    kTailNone = 0,
    kTailNormQuant = 1,  // rmsnorm(out) + quantize into tail_xq/xs               (qwen.c:569-570)
    kTailNextToken = 3,  // the prompt's next token or head_ids[argmax]            (qwen.c:677-683)
};

struct DecodeParams {
    const uint8_t *w[3];
    const uint16_t *ws[3];
    int rows[3];        // rows of each matrix; the output row space is their concatenation (or the pair)
    int n, rt, d;       // columns, output rows per tile, output rows in total
    const int8_t *xq;   // quantized input (n) and its scales (n/32) (kProQuantized)
    const float *xs;
    const float *src;   // fp32 input (kProQuant, kProNorm) and the rmsnorm weight (kProNorm)
    const float *norm_w;
    float *out;
    State *st;
    ExpTable et;
    int *counter;
    const float *tail_norm;  // rmsnorm weight of the tail
    float eps;
    int8_t *tail_xq;
    float *tail_xs;
    const int *prompt;
    const int32_t *head_ids;
    int *ids;
    int cap;
};

template <int BITS, int EPI, int PRO, int TAIL, int UPT>
__global__ void __launch_bounds__(kThreads) decode_matvec_kernel(const DecodeParams p) {
    constexpr int GB = BITS == 4 ? 16 : 32;
    constexpr int WC = GB / 16;
    extern __shared__ __align__(16) uint8_t smem[];
    const int n = p.n, ng = n / 32, tid = threadIdx.x;
    const int row0 = blockIdx.x * p.rt;
    const int rows = min(p.rt, p.d - row0);
    const int vrows = EPI == kEpiSwiGLU ? 2 * rows : rows;
    const int units = vrows * ng;

    // 1. this tile's weights and scales into registers: they do not depend on any earlier kernel
    uint4 wv[UPT][WC];
    uint32_t hs[UPT];
#pragma unroll
    for (int k = 0; k < UPT; k++) {
        const int u = tid + k * kThreads;
        if (u < units) {
            const int vr = u / ng, g = u - vr * ng;
            int m, r;
            if (EPI == kEpiSwiGLU) {
                m = vr < rows ? 0 : 1;
                r = row0 + (vr < rows ? vr : vr - rows);
            } else {
                r = row0 + vr;
                m = 0;
                if (r >= p.rows[0]) { r -= p.rows[0]; m = 1; }
                if (m == 1 && r >= p.rows[1]) { r -= p.rows[1]; m = 2; }
            }
            const uint8_t *wb = m == 0 ? p.w[0] : (m == 1 ? p.w[1] : p.w[2]);
            const uint16_t *sb = m == 0 ? p.ws[0] : (m == 1 ? p.ws[1] : p.ws[2]);
            const size_t idx = (size_t)r * ng + g;
#pragma unroll
            for (int c = 0; c < WC; c++) wv[k][c] = ld_weights(wb + idx * GB + 16 * c);
            hs[k] = ld_u16(sb + idx);
        }
    }
    allow_consumer();
    wait_for_producer();

    // 2. this kernel's int8 input in shared-memory planes: from the previous kernel's int8 output, or quantized
    //    (after an rmsnorm) from its fp32 output by this CTA
    uint4 *xplane = reinterpret_cast<uint4 *>(smem);
    float *xs_s = reinterpret_cast<float *>(xplane + 2 * ng);
    int *xsum_s = reinterpret_cast<int *>(xs_s + ng);
    float *prod = reinterpret_cast<float *>(xsum_s + ng);
    auto put_chunk = [&](int g, int k, uint4 a) {  // 16 activation bytes (chunk k of group g) into the planes
        if (BITS == 4) {
            uint32_t *ev = reinterpret_cast<uint32_t *>(&xplane[g]) + 2 * k;
            uint32_t *od = reinterpret_cast<uint32_t *>(&xplane[ng + g]) + 2 * k;
            ev[0] = __byte_perm(a.x, a.y, 0x6420);
            ev[1] = __byte_perm(a.z, a.w, 0x6420);
            od[0] = __byte_perm(a.x, a.y, 0x7531);
            od[1] = __byte_perm(a.z, a.w, 0x7531);
        } else {
            xplane[k * ng + g] = a;
        }
    };
    if (PRO == kProQuantized) {
        for (int c = tid; c < n / 16; c += kThreads) put_chunk(c >> 1, c & 1, __ldcg(reinterpret_cast<const uint4 *>(p.xq) + c));
        for (int g = tid; g < ng; g += kThreads) xs_s[g] = __ldcg(p.xs + g);
    } else {
        const float *src = p.src;
        if (PRO == kProNorm) {  // x and the normalized x live after the product stage
            float *xv = prod + (size_t)(EPI == kEpiSwiGLU ? 2 * p.rt : p.rt) * (ng + 1);
            xv = reinterpret_cast<float *>((reinterpret_cast<uintptr_t>(xv) + 15) & ~(uintptr_t)15);
            for (int j = tid; j < n / 4; j += kThreads) reinterpret_cast<float4 *>(xv)[j] = ld_cg4(p.src + 4 * j);
            __shared__ float s_inv;
            __syncthreads();
            if (tid == 0) {
                float ss = sum_squares_inorder(xv, n);
                ss = __fdiv_rn(ss, (float)n);
                ss = __fadd_rn(ss, p.eps);
                s_inv = __fdiv_rn(1.0f, __fsqrt_rn(ss));
            }
            __syncthreads();
            const float sc = s_inv;
            for (int j = tid; j < n; j += kThreads) xv[n + j] = __fmul_rn(p.norm_w[j], __fmul_rn(sc, xv[j]));
            __syncthreads();
            src = xv + n;
        }
        for (int g = tid; g < ng; g += kThreads) {
            int8_t q[32];
            float v[32];
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const float4 f = PRO == kProNorm ? reinterpret_cast<const float4 *>(src + 32 * g)[i]
                                                 : ld_cg4(src + 32 * g + 4 * i);
                v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
            }
            xs_s[g] = quantize32_qwen(v, q);
            uint32_t w[8];
#pragma unroll
            for (int j = 0; j < 8; j++)
                w[j] = (uint32_t)(uint8_t)q[4 * j] | (uint32_t)(uint8_t)q[4 * j + 1] << 8 |
                       (uint32_t)(uint8_t)q[4 * j + 2] << 16 | (uint32_t)(uint8_t)q[4 * j + 3] << 24;
            put_chunk(g, 0, make_uint4(w[0], w[1], w[2], w[3]));
            put_chunk(g, 1, make_uint4(w[4], w[5], w[6], w[7]));
        }
    }
    __syncthreads();
    if (BITS == 4) {
        for (int g = tid; g < ng; g += kThreads) {
            const uint4 e = xplane[g], o = xplane[ng + g];
            int s = __dp4a((int)e.x, 0x01010101, 0);
            s = __dp4a((int)e.y, 0x01010101, s);
            s = __dp4a((int)e.z, 0x01010101, s);
            s = __dp4a((int)e.w, 0x01010101, s);
            s = __dp4a((int)o.x, 0x01010101, s);
            s = __dp4a((int)o.y, 0x01010101, s);
            s = __dp4a((int)o.z, 0x01010101, s);
            s = __dp4a((int)o.w, 0x01010101, s);
            xsum_s[g] = s;
        }
        __syncthreads();
    }

    // 3. group products (matvec_kernel's arithmetic)
#pragma unroll
    for (int k = 0; k < UPT; k++) {
        const int u = tid + k * kThreads;
        if (u < units) {
            const int vr = u / ng, g = u - vr * ng;
            int acc = 0;
            if (BITS == 4) {
                const uint4 e = xplane[g], o = xplane[ng + g];
                const uint32_t w4[4] = {wv[k][0].x, wv[k][0].y, wv[k][0].z, wv[k][0].w};
                const uint32_t ev[4] = {e.x, e.y, e.z, e.w}, ov[4] = {o.x, o.y, o.z, o.w};
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const uint32_t lo = (w4[j] & 0x0F0F0F0Fu) ^ 0x08080808u;
                    const uint32_t hi = ((w4[j] >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
                    acc = __dp4a((int)lo, (int)ev[j], acc);
                    acc = __dp4a((int)hi, (int)ov[j], acc);
                }
                acc -= 8 * xsum_s[g];
            } else {
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    const uint4 a = xplane[c * ng + g];
                    acc = __dp4a((int)wv[k][c].x, (int)a.x, acc);
                    acc = __dp4a((int)wv[k][c].y, (int)a.y, acc);
                    acc = __dp4a((int)wv[k][c].z, (int)a.z, acc);
                    acc = __dp4a((int)wv[k][c].w, (int)a.w, acc);
                }
            }
            prod[vr * (ng + 1) + g] = __fmul_rn(__fmul_rn(__int2float_rn(acc), scale_from_f16(hs[k])), xs_s[g]);
        }
    }
    __syncthreads();

    // 4. in-order fold of each virtual row, epilogue
    float v = 0.0f;
    if (tid < vrows) {
        const float *pr = prod + tid * (ng + 1);
#pragma unroll 8
        for (int j = 0; j < ng; j++) v = __fadd_rn(v, pr[j]);
    }
    if (EPI == kEpiStore) {
        if (tid < rows) p.out[row0 + tid] = v;
    } else if (EPI == kEpiResidual) {
        if (tid < rows) p.out[row0 + tid] = __fadd_rn(__ldcg(p.out + row0 + tid), v);
    } else if (EPI == kEpiSwiGLU) {
        __syncthreads();  // prod is reused for the fold values
        if (tid < vrows) prod[tid] = v;
        __syncthreads();
        if (tid < rows) {
            float gv = prod[tid];
            const float u = prod[rows + tid];
            gv = __fmul_rn(gv, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf_ref(-gv, p.et))));
            p.out[row0 + tid] = __fmul_rn(gv, u);
        }
    } else {  // kEpiHead
        unsigned long long key = 0ull;
        if (tid < rows) {
            p.out[row0 + tid] = v;
            const float c = v == 0.0f ? 0.0f : v;  // -0 ties with +0, as the reference's `>` sees them
            const uint32_t b = __float_as_uint(c);
            const uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
            if (c == c) key = ((unsigned long long)ord << 32) | (uint32_t)(~(uint32_t)(row0 + tid));
        }
#pragma unroll
        for (int off = 16; off; off >>= 1) {
            const unsigned long long o = __shfl_xor_sync(0xffffffffu, key, off);
            key = o > key ? o : key;
        }
        if ((tid & 31) == 0 && key) atomicMax(&p.st->key, key);
    }

    // 5. the last CTA prepares the next kernel's input
    if (TAIL == kTailNone || !last_cta(p.counter)) return;
    float *sm = reinterpret_cast<float *>(smem);
    if (TAIL == kTailNormQuant) {
        for (int j = tid; j < p.d / 4; j += kThreads) reinterpret_cast<float4 *>(sm)[j] = ld_cg4(p.out + 4 * j);
        rmsnorm_quantize(sm, sm + p.d, p.tail_norm, p.eps, p.d, p.tail_xq, p.tail_xs);
    } else if (TAIL == kTailNextToken && tid == 0) {
        State *st = p.st;
        const int pos = st->pos;
        const unsigned long long key = atomicAdd(&st->key, 0ull);
        // no key: every logit was NaN; the reference's strict `>` then keeps row 0 (qwen.c:591-598)
        const int row = key ? (int)(~(uint32_t)(key & 0xffffffffu)) : 0;
        st->last_row = row;
        if (st->n_prompt >= 0) {
            int next;
            if (pos + 1 < st->n_prompt) {
                next = p.prompt[pos + 1];
            } else {
                next = p.head_ids[row];
                if (st->n_gen < p.cap) p.ids[st->n_gen] = next;
                st->n_gen++;
            }
            st->token = next;
        }
        st->pos = pos + 1;
    }
}

// Dynamic shared memory of decode_matvec_kernel: the product stage (plus x and the normalized x for an rmsnorm
// prologue), or the tail's staging if larger.
inline size_t decode_smem_bytes(int n, int rt, int epi, int pro, int tail, int d) {
    const int ng = n / 32;
    const int vmax = epi == kEpiSwiGLU ? 2 * rt : rt;
    size_t b = (size_t)2 * ng * 16 + (size_t)ng * 8 + (size_t)vmax * (ng + 1) * 4;
    if (pro == kProNorm) b = ((b + 15) & ~(size_t)15) + (size_t)2 * n * 4;
    size_t t = tail == kTailNormQuant ? (size_t)2 * d * 4 : 0;
    return b > t ? b : t;
}

// ---------------------------------------------------------------------------------------------------------------
// attention for one query head (qwen.c:521-546): biases, NeoX RoPE (pairs i, i + hs/2), the KV-cache write of
// this position, scores q.k / sqrt(hs) in order over the head's elements, softmax in order, weighted values in
// order of position. The cached values of this head's kv head are staged in shared memory (cp.async, double
// buffered in chunks of kVChunk positions) while the scores are computed. The last CTA quantizes the output.
constexpr int kVChunk = 128;

struct AttnParams {
    const float *qkv;   // raw outputs of the qkv matvec: q (dim) | k (kv_dim) | v (kv_dim)
    const float *bq, *bk, *bv;
    const float *rope;  // per position: cos[hs/2] then sin[hs/2]
    float *kcache, *vcache;  // this layer's (ctx, kv_dim)
    float *xb;          // dim outputs
    int dim, kv_dim, kv_mul, ctx;
    State *st;
    ExpTable et;
};

__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gmem_src) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem_dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <int HS>
__device__ __forceinline__ void stage_values(float *dst, const float *vcache, int kv_dim, int kvh, int t0, int nt) {
    // rows t0 .. t0+nt-1 of this kv head, HS floats each: HS/4 16-byte pieces per row
    for (int c = threadIdx.x; c < nt * (HS / 4); c += blockDim.x) {
        const int t = c / (HS / 4), q = c % (HS / 4);
        cp_async16(dst + t * HS + 4 * q, vcache + (size_t)(t0 + t) * kv_dim + kvh * HS + 4 * q);
    }
}

template <int HS>
__global__ void __launch_bounds__(kThreads) attention_kernel(const AttnParams p) {
    extern __shared__ __align__(16) float asm_[];
    float *q = asm_, *kc = q + HS, *vc = kc + HS;
    float *att = vc + HS;                                  // ctx scores
    float *vbuf = att + ((p.ctx + 3) & ~3);                // 2 x kVChunk x HS staged values
    __shared__ float red[kThreads / 32];
    __shared__ float s_max, s_sum;
    const int h = blockIdx.x, kvh = h / p.kv_mul, half = HS / 2, tid = threadIdx.x;
    allow_consumer();
    wait_for_producer();
    const int pos = __ldcg(&p.st->pos);
    const int nchunks = (pos + kVChunk - 1) / kVChunk;  // cached positions 0 .. pos-1
    if (nchunks > 0) stage_values<HS>(vbuf, p.vcache, p.kv_dim, kvh, 0, min(kVChunk, pos));
    cp_async_commit();
    // this thread's first cached key row, loaded before the rope so both round trips overlap
    float4 k4[HS / 4];
    if (tid < pos) {
        const float *kt = p.kcache + (size_t)tid * p.kv_dim + kvh * HS;
#pragma unroll
        for (int i = 0; i < HS / 4; i++) k4[i] = ld_cg4(kt + 4 * i);
    }
    const float *cs = p.rope + (size_t)pos * HS;
    const float *qr = p.qkv + h * HS, *kr = p.qkv + p.dim + kvh * HS, *vr = p.qkv + p.dim + p.kv_dim + kvh * HS;
    if (tid < half) {
        const float c = cs[tid], s = cs[half + tid];
        float a = __fadd_rn(__ldcg(qr + tid), p.bq[h * HS + tid]);
        float b = __fadd_rn(__ldcg(qr + tid + half), p.bq[h * HS + tid + half]);
        q[tid] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
        q[tid + half] = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
        a = __fadd_rn(__ldcg(kr + tid), p.bk[kvh * HS + tid]);
        b = __fadd_rn(__ldcg(kr + tid + half), p.bk[kvh * HS + tid + half]);
        kc[tid] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
        kc[tid + half] = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
    }
    if (tid < HS) vc[tid] = __fadd_rn(__ldcg(vr + tid), p.bv[kvh * HS + tid]);
    __syncthreads();
    if (h % p.kv_mul == 0 && tid < HS) {  // one writer per kv head
        p.kcache[(size_t)pos * p.kv_dim + kvh * HS + tid] = kc[tid];
        p.vcache[(size_t)pos * p.kv_dim + kvh * HS + tid] = vc[tid];
    }
    // scores: one position per thread, the head's HS products added in order
    const float scale = __fsqrt_rn((float)HS);
    for (int t = tid; t <= pos; t += kThreads) {
        if (t == pos) {
#pragma unroll
            for (int i = 0; i < HS / 4; i++) k4[i] = reinterpret_cast<const float4 *>(kc)[i];
        } else if (t != tid) {
            const float *kt = p.kcache + (size_t)t * p.kv_dim + kvh * HS;
#pragma unroll
            for (int i = 0; i < HS / 4; i++) k4[i] = ld_cg4(kt + 4 * i);
        }
        float score = 0.0f;
#pragma unroll
        for (int i = 0; i < HS / 4; i++) {
            score = __fadd_rn(score, __fmul_rn(q[4 * i], k4[i].x));
            score = __fadd_rn(score, __fmul_rn(q[4 * i + 1], k4[i].y));
            score = __fadd_rn(score, __fmul_rn(q[4 * i + 2], k4[i].z));
            score = __fadd_rn(score, __fmul_rn(q[4 * i + 3], k4[i].w));
        }
        att[t] = __fdiv_rn(score, scale);
    }
    __syncthreads();
    // softmax (qwen.c:346-352): max, exp(x - max), in-order sum, divide
    float m = -INFINITY;
    for (int t = tid; t <= pos; t += kThreads) m = fmaxf(m, att[t]);
#pragma unroll
    for (int off = 16; off; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if ((tid & 31) == 0) red[tid >> 5] = m;
    __syncthreads();
    if (tid == 0) {
        float mm = red[0];
        for (int w = 1; w < kThreads / 32; w++) mm = fmaxf(mm, red[w]);
        s_max = mm;
    }
    __syncthreads();
    const float mx = s_max;
    for (int t = tid; t <= pos; t += kThreads) att[t] = expf_ref(__fsub_rn(att[t], mx), p.et);
    __syncthreads();
    if (tid == 0) s_sum = sum_inorder(att, pos + 1);
    __syncthreads();
    const float sum = s_sum;
    for (int t = tid; t <= pos; t += kThreads) att[t] = __fdiv_rn(att[t], sum);
    // weighted values, in order of position, from the staged chunks
    float acc = 0.0f;
    for (int c = 0; c < nchunks; c++) {
        if (c + 1 < nchunks) {
            const int t0 = (c + 1) * kVChunk;
            stage_values<HS>(vbuf + ((c + 1) & 1) * kVChunk * HS, p.vcache, p.kv_dim, kvh, t0, min(kVChunk, pos - t0));
        }
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        if (tid < HS) {
            const float *vb = vbuf + (c & 1) * kVChunk * HS + tid;
            const int t0 = c * kVChunk, nt = min(kVChunk, pos - t0);
#pragma unroll 8
            for (int t = 0; t < nt; t++) acc = __fadd_rn(acc, __fmul_rn(att[t0 + t], vb[t * HS]));
        }
        __syncthreads();
    }
    if (tid < HS) {
        acc = __fadd_rn(acc, __fmul_rn(att[pos], vc[tid]));
        p.xb[h * HS + tid] = acc;
    }
}

template <int HS>
inline size_t attention_smem_bytes(int ctx) {
    return (size_t)3 * HS * 4 + (size_t)((ctx + 3) & ~3) * 4 + (size_t)2 * kVChunk * HS * 4;
}

}  // namespace qwen
}  // namespace mvb
