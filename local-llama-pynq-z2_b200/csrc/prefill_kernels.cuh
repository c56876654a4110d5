// Kernels of the batched prompt prefill (qwen_decode.cu, mvb_qwen_prefill): the decode step's per-token
// arithmetic (decode_kernels.cuh, itself qwen.c's, operation by operation) applied to M prompt tokens at once, with
// the matvecs done by the tensor-core matmul of gemm.cu, which is bit-identical to the matvec for every token.
// One CTA per token row (or per token and head for the attention); the KV-cache rows they write are the ones
// the decode step would have written for those positions, so decoding continues from them unchanged.
//
// Activations for the matmul: xq is token-major (row t holds token t's n int8 values), xs group-major
// (xs[g * ldx + t] is token t's scale of group g).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "decode_kernels.cuh"
#include "expf_ref.h"
#include "matvec_kernels.cuh"

namespace mvb {
namespace decode {

// Quantizes v[0 .. n-1] (shared memory, 16-byte aligned) per group of 32 like qwen.c:355-364 into xq (element
// order) and xs[g * ldx]; the operations of quantize_to_planes, with eight threads per group. Whole CTA of
// kThreads threads (every thread takes the same number of passes: the shuffles need the full warp).
__device__ __forceinline__ void quantize_row(const float *v, int n, int8_t *xq, float *xs, int ldx) {
    const int ng = n / 32, l = threadIdx.x & 7;
    for (int base = 0; base < ng; base += kThreads / 8) {
        const int g = base + (threadIdx.x >> 3);
        const bool on = g < ng;
        float4 f = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (on) f = reinterpret_cast<const float4 *>(v + 32 * g)[l];
        auto bits = [](float x) {
            const float a = fabsf(x);
            return a == a ? __float_as_uint(a) : 0u;
        };
        unsigned m = max(max(bits(f.x), bits(f.y)), max(bits(f.z), bits(f.w)));
        m = max(m, __shfl_xor_sync(0xffffffffu, m, 1));
        m = max(m, __shfl_xor_sync(0xffffffffu, m, 2));
        m = max(m, __shfl_xor_sync(0xffffffffu, m, 4));
        const float scale = __fmul_rn(__uint_as_float(m), 1.0f / 127.0f);
        const float inv = scale > 0.0f ? __frcp_rn(scale) : 0.0f;
        const uint32_t q0 = (uint8_t)to_int8_x86(roundf(__fmul_rn(f.x, inv)));
        const uint32_t q1 = (uint8_t)to_int8_x86(roundf(__fmul_rn(f.y, inv)));
        const uint32_t q2 = (uint8_t)to_int8_x86(roundf(__fmul_rn(f.z, inv)));
        const uint32_t q3 = (uint8_t)to_int8_x86(roundf(__fmul_rn(f.w, inv)));
        if (on) {
            *reinterpret_cast<uint32_t *>(xq + 32 * g + 4 * l) = q0 | q1 << 8 | q2 << 16 | q3 << 24;
            if (l == 0) xs[(size_t)g * ldx] = scale;
        }
    }
}

// x[t] = dequantized embedding row of tokens[t] (embed_kernel's arithmetic).
__global__ void embed_rows_kernel(const int8_t *emb_q, const uint16_t *emb_s, const int *tokens, float *x, int dim) {
    const int t = blockIdx.x;
    const size_t r = (size_t)tokens[t] * dim;
    for (int i = threadIdx.x; i < dim; i += blockDim.x)
        x[(size_t)t * dim + i] = __fmul_rn(__int2float_rn(emb_q[r + i]), scale_from_f16(emb_s[r / 32 + i / 32]));
}

// rmsnorm (qwen.c:337-344) of row t of x with weight w, then quantize: decode_matvec_kernel's kProNorm prologue;
// with `add`, row t of add is first added into x (the residual of the matmul before). Dynamic shared memory: 2n
// floats.
__global__ void __launch_bounds__(kThreads) norm_quant_rows_kernel(float *x, const float *add, const float *w,
                                                                   float eps, int n, int8_t *xq, float *xs, int ldx) {
    extern __shared__ __align__(16) float sm[];
    float *xv = sm, *xn = sm + n;
    __shared__ float s_inv;
    const int t = blockIdx.x;
    float *xr = x + (size_t)t * n;
    // with `add`, the residual add of the matmul just before (qwen.c:551, :565) comes first: x += add, stored back
    const float *ar = add ? add + (size_t)t * n : nullptr;
    for (int j = threadIdx.x; j < n / 4; j += kThreads) {
        float4 f = ld_cg4(xr + 4 * j);
        if (ar) {
            const float4 a = ld_cg4(ar + 4 * j);
            f = make_float4(__fadd_rn(f.x, a.x), __fadd_rn(f.y, a.y), __fadd_rn(f.z, a.z), __fadd_rn(f.w, a.w));
            reinterpret_cast<float4 *>(xr)[j] = f;
        }
        reinterpret_cast<float4 *>(xv)[j] = f;
    }
    __syncthreads();
    for (int j = threadIdx.x; j < n; j += kThreads) xn[j] = __fmul_rn(xv[j], xv[j]);
    __syncthreads();
    if (threadIdx.x == 0) {
        float ss = chain_sum(xn, n);
        ss = __fdiv_rn(ss, (float)n);
        ss = __fadd_rn(ss, eps);
        s_inv = __frcp_rn(__fsqrt_rn(ss));  // 1.0f / sqrtf(...): the correctly rounded reciprocal
    }
    __syncthreads();
    const float sc = s_inv;
    for (int j = threadIdx.x; j < n; j += kThreads) xn[j] = __fmul_rn(w[j], __fmul_rn(sc, xv[j]));
    __syncthreads();
    quantize_row(xn, n, xq + (size_t)t * n, xs + t, ldx);
}

// quantize row t of src (qwen.c:355-364): the kProQuant prologue. Dynamic shared memory: n floats.
__global__ void __launch_bounds__(kThreads) quant_rows_kernel(const float *src, int n, int8_t *xq, float *xs, int ldx) {
    extern __shared__ __align__(16) float sm[];
    const int t = blockIdx.x;
    const float *sr = src + (size_t)t * n;
    for (int j = threadIdx.x; j < n / 4; j += kThreads) reinterpret_cast<float4 *>(sm)[j] = ld_cg4(sr + 4 * j);
    __syncthreads();
    quantize_row(sm, n, xq + (size_t)t * n, xs + t, ldx);
}

// SwiGLU of rows t = blockIdx.x of h1 (gate) and h3 (up) (qwen.c:558-562, the kEpiSwiGLU epilogue), then quantize
// (the down projection's kProQuant prologue), for the groups [32 * blockIdx.y, 32 * blockIdx.y + 32) of the row:
// groups are independent, so a token's row is spread over several CTAs. Static shared memory: 32 groups.
__global__ void __launch_bounds__(kThreads) swiglu_quant_rows_kernel(const float *h1, const float *h3, int n,
                                                                     ExpTable et, int8_t *xq, float *xs, int ldx) {
    __shared__ __align__(16) float sm[32 * 32];
    const int t = blockIdx.x, g0 = blockIdx.y * 32, ng = min(32, n / 32 - g0), e0 = g0 * 32;
    for (int j = threadIdx.x; j < ng * 32; j += kThreads) {
        float gv = __ldcg(h1 + (size_t)t * n + e0 + j);
        const float u = __ldcg(h3 + (size_t)t * n + e0 + j);
        gv = __fmul_rn(gv, __frcp_rn(__fadd_rn(1.0f, expf_ref(-gv, et))));  // 1.0f / (...) of qwen.c
        sm[j] = __fmul_rn(gv, u);
    }
    __syncthreads();
    quantize_row(sm, ng * 32, xq + (size_t)t * n + e0, xs + (size_t)g0 * ldx + t, ldx);
}

// x += add, element by element (the kEpiResidual epilogue: x = x + matvec).
__global__ void residual_rows_kernel(float *x, const float *add, size_t count) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (size_t)gridDim.x * blockDim.x)
        x[i] = __fadd_rn(x[i], add[i]);
}

// Biases, NeoX RoPE and the KV-cache write for the token of row t at position p0 + t (attention_kernel's
// prologue): q rows go to qb, k and v rows to the caches.
__global__ void rope_cache_rows_kernel(const float *qkv, int ldq, const float *bq, const float *bk, const float *bv,
                                       const float *rope, float *kcache, float *vcache, float *qb, int p0, int dim,
                                       int kv_dim, int hs) {
    const int t = blockIdx.x, pos = p0 + t, half = hs / 2;
    const float *cs = rope + (size_t)pos * hs;
    const float *row = qkv + (size_t)t * ldq;
    const int nq = dim / 2, nk = kv_dim / 2;  // rotated pairs of q and of k
    for (int u = threadIdx.x; u < nq + nk + kv_dim; u += blockDim.x) {
        if (u < nq + nk) {
            const bool isq = u < nq;
            const int p = isq ? u : u - nq;            // pair index
            const int h = p / half, i = p % half;      // head, element
            const float *src = isq ? row : row + dim;
            const float *b = isq ? bq : bk;
            const int e0 = h * hs + i, e1 = e0 + half;
            const float c = cs[i], s = cs[half + i];
            const float a = __fadd_rn(src[e0], b[e0]);
            const float bb = __fadd_rn(src[e1], b[e1]);
            const float r0 = __fsub_rn(__fmul_rn(a, c), __fmul_rn(bb, s));
            const float r1 = __fadd_rn(__fmul_rn(bb, c), __fmul_rn(a, s));
            if (isq) {
                qb[(size_t)t * dim + e0] = r0;
                qb[(size_t)t * dim + e1] = r1;
            } else {
                kcache[(size_t)pos * kv_dim + e0] = r0;
                kcache[(size_t)pos * kv_dim + e1] = r1;
            }
        } else {
            const int e = u - nq - nk;
            vcache[(size_t)pos * kv_dim + e] = __fadd_rn(row[dim + kv_dim + e], bv[e]);
        }
    }
}

// Attention of the token of row t = blockIdx.x (position p0 + t) for query head blockIdx.y, over the cache rows
// 0 .. p0 + t (qwen.c:521-546): attention_kernel's scores, softmax and weighted values, operation by operation.
// Dynamic shared memory: attention_rows_smem_bytes.
template <int HS>
__global__ void __launch_bounds__(kThreads) attention_rows_kernel(const float *qb, const float *kcache,
                                                                  const float *vcache, float *out, int p0, int dim,
                                                                  int kv_dim, int kv_mul, int npos, int vchunk,
                                                                  ExpTable et) {
    extern __shared__ __align__(16) float asm_[];
    float *q = asm_;
    float *att = q + HS;                    // scores of positions 0 .. npos-1 (npos = the batch's last position + 1)
    float *vbuf = att + ((npos + 3) & ~3);  // vchunk x HS staged values
    __shared__ float red[kThreads / 32];
    __shared__ float s_max, s_sum;
    const int t = blockIdx.x, h = blockIdx.y, kvh = h / kv_mul, tid = threadIdx.x, pos = p0 + t;
    if (tid < HS) q[tid] = qb[(size_t)t * dim + h * HS + tid];
    __syncthreads();
    const float scale = __fsqrt_rn((float)HS);
    for (int u = tid; u <= pos; u += kThreads) {
        const float *kt = kcache + (size_t)u * kv_dim + kvh * HS;
        float4 k4[HS / 4];
#pragma unroll
        for (int i = 0; i < HS / 4; i++) k4[i] = ld_cg4(kt + 4 * i);
        float score = 0.0f;
#pragma unroll
        for (int i = 0; i < HS / 4; i++) {
            score = __fadd_rn(score, __fmul_rn(q[4 * i], k4[i].x));
            score = __fadd_rn(score, __fmul_rn(q[4 * i + 1], k4[i].y));
            score = __fadd_rn(score, __fmul_rn(q[4 * i + 2], k4[i].z));
            score = __fadd_rn(score, __fmul_rn(q[4 * i + 3], k4[i].w));
        }
        att[u] = __fdiv_rn(score, scale);
    }
    __syncthreads();
    float m = -INFINITY;
    for (int u = tid; u <= pos; u += kThreads) m = fmaxf(m, att[u]);
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
    for (int u = tid; u <= pos; u += kThreads) att[u] = expf_ref(__fsub_rn(att[u], mx), et);
    __syncthreads();
    if (tid == 0) s_sum = chain_sum(att, pos + 1);
    __syncthreads();
    const float sum = s_sum;
    for (int u = tid; u <= pos; u += kThreads) att[u] = __fdiv_rn(att[u], sum);
    // weighted values of the cached positions 0 .. pos-1 in order, then this position's
    float acc = 0.0f;
    for (int t0 = 0; t0 < pos; t0 += vchunk) {
        const int nt = min(vchunk, pos - t0);
        __syncthreads();  // the previous chunk has been read
        stage_values<HS>(vbuf, vcache, kv_dim, kvh, t0, nt);
        cp_async_commit();
        cp_async_wait<0>();
        __syncthreads();
        if (tid < HS) acc = weighted_chain<HS>(acc, att + t0, vbuf + tid, nt);
    }
    if (tid < HS) {
        acc = __fadd_rn(acc, __fmul_rn(att[pos], vcache[(size_t)pos * kv_dim + kvh * HS + tid]));
        out[(size_t)t * dim + h * HS + tid] = acc;
    }
}

// Shared memory of attention_rows_kernel for positions 0 .. npos-1 and value chunks of vchunk positions.
template <int HS>
inline size_t attention_rows_smem_bytes(int npos, int vchunk) {
    return (size_t)HS * 4 + (size_t)((npos + 3) & ~3) * 4 + (size_t)vchunk * HS * 4;
}

// acc_lo = ((0 + a_0 v_0) + a_1 v_1) + ... over t < nt in order, and acc_hi the same for the value beside it: two
// independent in-order chains (values at vb + t * HS and vb + t * HS + 1; vb 8-byte aligned, a 16-byte aligned).
// The products of a block of 8 positions are formed one block ahead of their adds.
template <int HS>
__device__ __forceinline__ float2 weighted_chain_pair(const float *a, const float *vb, int nt) {
    float2 acc = make_float2(0.0f, 0.0f);
    const int n8 = nt & ~7;
    auto form = [&](int t0, float2 (&p)[8]) {
        const float4 a0 = *reinterpret_cast<const float4 *>(a + t0), a1 = *reinterpret_cast<const float4 *>(a + t0 + 4);
        const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const float2 v = *reinterpret_cast<const float2 *>(vb + (t0 + i) * HS);
            p[i] = make_float2(__fmul_rn(av[i], v.x), __fmul_rn(av[i], v.y));
        }
    };
    float2 p[8];
    if (n8 > 0) form(0, p);
    for (int t = 0; t < n8; t += 8) {
        float2 nx[8];
        form(t + 8 < n8 ? t + 8 : t, nx);  // stays inside [0, n8)
#pragma unroll
        for (int i = 0; i < 8; i++) {
            acc.x = __fadd_rn(acc.x, p[i].x);
            acc.y = __fadd_rn(acc.y, p[i].y);
        }
#pragma unroll
        for (int i = 0; i < 8; i++) p[i] = nx[i];
    }
    for (int t = n8; t < nt; t++) {
        const float av = a[t];
        const float2 v = *reinterpret_cast<const float2 *>(vb + t * HS);
        acc.x = __fadd_rn(acc.x, __fmul_rn(av, v.x));
        acc.y = __fadd_rn(acc.y, __fmul_rn(av, v.y));
    }
    return acc;
}

// The same causal attention (qwen.c:521-546) with the keys and values shared by the query heads of a group: one CTA
// per (token t,
// kv head) and one warp per query head of the group (kv_mul warps). The kv head's keys and values of positions
// 0 .. pos are staged into shared memory once (16-byte cp.async pieces) and read by every warp, where
// attention_rows_kernel has each of the kv_mul query-head CTAs read them from L2 on its own. Per query head the
// arithmetic is attention_rows_kernel's, operation for operation, so the outputs are the same bits:
//   scores   s_u = ((0 + q_0 k_u0) + q_1 k_u1) + ... in dimension order, then s_u / sqrt(HS)   (lane: u = lane + 32i,
//            four positions at a time)
//   softmax  max (order-free), expf_ref(s_u - max), the sum in position order (lane 0), then s_u / sum
//   values   o_d = ((0 + a_0 v_0d) + a_1 v_1d) + ... + a_pos v_pos,d in position order     (lane: d = 2 lane, 2 lane + 1)
// and then, in place of quant_rows_kernel, the quantization of the head's 64 outputs for the o projection: they are
// whole groups of 32 (lanes 0-15 and 16-31), quantized with quantize_row's operations (qwen.c:355-364) into xq
// (token-major) and xs (group-major, ldx). The key rows are padded to HS + 4 floats: the float4 reads of eight
// consecutive lanes (eight consecutive rows) then fall in eight different 16-byte bank groups. Shared memory:
// attention_gqa_smem_bytes(npos, kv_mul).
template <int HS>
__global__ void __launch_bounds__(1024) attention_gqa_rows_kernel(const float *qb, const float *kcache,
                                                                   const float *vcache, int8_t *xq, float *xs, int ldx,
                                                                   int p0, int dim, int kv_dim, int kv_mul, int npos,
                                                                   ExpTable et) {
    static_assert(HS == 64, "two values per lane, two quantization groups per head");
    constexpr int KS = HS + 4;
    extern __shared__ __align__(16) float gsm[];
    const int t = blockIdx.x, kvh = blockIdx.y, pos = p0 + t, tid = threadIdx.x;
    const int npad = (npos + 3) & ~3;
    float *ks = gsm;                          // [npos][KS] keys
    float *vs = ks + (size_t)npos * KS;       // [npos][HS] values
    float *att = vs + (size_t)npos * HS;      // [kv_mul][npad] scores, then weights
    float *qs = att + (size_t)kv_mul * npad;  // [kv_mul][HS] the group's queries
    for (int c = tid; c < (pos + 1) * (HS / 4); c += blockDim.x) {
        const int u = c / (HS / 4), k = c % (HS / 4);
        const size_t g = (size_t)u * kv_dim + kvh * HS + 4 * k;
        cp_async16(ks + u * KS + 4 * k, kcache + g);
        cp_async16(vs + u * HS + 4 * k, vcache + g);
    }
    cp_async_commit();
    for (int c = tid; c < kv_mul * HS; c += blockDim.x) qs[c] = qb[(size_t)t * dim + (size_t)kvh * kv_mul * HS + c];
    cp_async_wait<0>();
    __syncthreads();
    const int w = tid >> 5, lane = tid & 31, h = kvh * kv_mul + w;
    const float *q = qs + w * HS;
    float *a = att + w * npad;
    const float scale = __fsqrt_rn((float)HS);
    float m = -INFINITY;
    for (int u0 = 0; u0 <= pos; u0 += 128) {
        int row[4];
        float sc[4];
#pragma unroll
        for (int r = 0; r < 4; r++) {
            const int u = u0 + 32 * r + lane;
            row[r] = u <= pos ? u : 0;  // past pos: row 0 (staged), result unused
            sc[r] = 0.0f;
        }
#pragma unroll 4
        for (int i = 0; i < HS; i += 4) {
            const float4 q4 = *reinterpret_cast<const float4 *>(q + i);
#pragma unroll
            for (int r = 0; r < 4; r++) {
                const float4 k4 = *reinterpret_cast<const float4 *>(ks + row[r] * KS + i);
                sc[r] = __fadd_rn(sc[r], __fmul_rn(q4.x, k4.x));
                sc[r] = __fadd_rn(sc[r], __fmul_rn(q4.y, k4.y));
                sc[r] = __fadd_rn(sc[r], __fmul_rn(q4.z, k4.z));
                sc[r] = __fadd_rn(sc[r], __fmul_rn(q4.w, k4.w));
            }
        }
#pragma unroll
        for (int r = 0; r < 4; r++) {
            const int u = u0 + 32 * r + lane;
            if (u <= pos) {
                const float v = __fdiv_rn(sc[r], scale);
                a[u] = v;
                m = fmaxf(m, v);
            }
        }
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    for (int u = lane; u <= pos; u += 32) a[u] = expf_ref(__fsub_rn(a[u], m), et);
    __syncwarp();
    float sum = 0.0f;
    if (lane == 0) sum = chain_sum(a, pos + 1);
    sum = __shfl_sync(0xffffffffu, sum, 0);
    for (int u = lane; u <= pos; u += 32) a[u] = __fdiv_rn(a[u], sum);
    __syncwarp();
    const float2 o = weighted_chain_pair<HS>(a, vs + 2 * lane, pos + 1);
    // quantize_row's operations on the group of lanes 0-15 (dims 0-31) and of lanes 16-31 (dims 32-63)
    auto bits = [](float x) {
        const float v = fabsf(x);
        return v == v ? __float_as_uint(v) : 0u;
    };
    unsigned mb = max(bits(o.x), bits(o.y));
#pragma unroll
    for (int off = 1; off < 16; off <<= 1) mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, off));
    const float qscale = __fmul_rn(__uint_as_float(mb), 1.0f / 127.0f);
    const float inv = qscale > 0.0f ? __frcp_rn(qscale) : 0.0f;
    const uint32_t q0 = (uint8_t)to_int8_x86(roundf(__fmul_rn(o.x, inv)));
    const uint32_t q1 = (uint8_t)to_int8_x86(roundf(__fmul_rn(o.y, inv)));
    *reinterpret_cast<uint16_t *>(xq + (size_t)t * dim + h * HS + 2 * lane) = (uint16_t)(q0 | q1 << 8);
    if ((lane & 15) == 0) xs[(size_t)(2 * h + (lane >> 4)) * ldx + t] = qscale;
}

// Shared memory of attention_gqa_rows_kernel for positions 0 .. npos-1 and kv_mul query heads per kv head.
template <int HS>
inline size_t attention_gqa_smem_bytes(int npos, int kv_mul) {
    return (size_t)npos * (2 * HS + 4) * 4 + (size_t)kv_mul * (((npos + 3) & ~3) + HS) * 4;
}

}  // namespace decode
}  // namespace mvb
