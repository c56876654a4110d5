// Device-resident Qwen2 decode over the group-quantized matvec (the reference's token loop, qwen/qwen.c:490-573
// and :669-712, moved onto the B200 so the matvecs run back to back instead of one host round trip each).
//
// One forward step is a fixed sequence of kernels, captured once into a CUDA graph:
//   embed                       x = dequantized embedding row of the current token          qwen.c:498-501
//   per layer:
//     qkv  (fused matvec)       rmsnorm(x) -> quantize -> [wq; wk; wv] rows, raw outputs     qwen.c:516-520
//     attention (per q head)    + biases, NeoX RoPE, KV-cache write, softmax attention       qwen.c:521-546
//     o    (fused matvec)       quantize(xb) -> wo, x += out                                 qwen.c:549-551
//     gate/up (fused matvec)    rmsnorm(x) -> quantize -> w1, w3 rows paired, SwiGLU -> hb    qwen.c:554-562
//     down (fused matvec)       quantize(hb) -> w2, x += out                                 qwen.c:563-565
//   final norm + quantize       rmsnorm(x) -> xq, xs                                         qwen.c:569-570
//   head (matvec)               Q8 head rows -> logits, block argmax -> atomicMax            qwen.c:571, 591-598
//   next token                  prompt[pos+1] while feeding the prompt, else head_ids[argmax] qwen.c:677-683
// The step reads the token and the position from device memory, so the same graph serves every position and
// a whole generation is the graph launched once per position with no host work in between.
//
// Arithmetic follows qwen.c operation by operation: no fused multiply-adds (the library is built with
// -fmad=false and uses explicitly rounded intrinsics), sums in the reference's order (rmsnorm's sum of squares,
// attention dots, the softmax denominator and the weighted value sum are all sequential loops there and here),
// RoPE angles from the host's double-precision pow/cos/sin exactly as qwen.c:504-508 computes them, and expf
// (softmax, SiLU) with the host C library's exact results (expf_ref.h), so the step reproduces qwen.c's logits
// bit for bit.
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include <map>
#include <mutex>
#include <vector>

#include "../../include/matvec_b200.h"
#include "expf_ref.h"
#include "matvec_kernels.cuh"
#include "mvb_runtime.h"

namespace mvb {
namespace qwen {

constexpr int kMaxDim = 2048;     // largest dim the fused prologues stage in shared memory
constexpr int kMaxHead = 128;     // largest head size of the attention kernel
constexpr int kMaxCtx = 8192;     // largest context (attention scores live in shared memory)
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


// ---------------------------------------------------------------------------------------------------------------
// embedding row (qwen.c:498-501): x[i] = er[i] * f16(es[i / 32]), exact in fp32
__global__ void embed_kernel(const int8_t *emb_q, const uint16_t *emb_s, float *x, int dim, State *st) {
    wait_for_producer();
    const int tok = st->token;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i == 0) st->key = 0ull;
    if (i < dim) {
        const size_t r = (size_t)tok * dim;
        x[i] = __fmul_rn(__int2float_rn(emb_q[r + i]), scale_from_f16(emb_s[r / 32 + i / 32]));
    }
    allow_consumer();
}

// ---------------------------------------------------------------------------------------------------------------
// rmsnorm of qwen.c:337-344 into shared memory: ss = sum x^2 in order, ss = 1/sqrtf(ss/n + eps), o = w * (ss * x).
// `sq` is n floats of scratch in shared memory; the sequential sum is one thread's loop, as in the reference.
__device__ void rmsnorm_smem(float *o, float *sq, const float *x, const float *w, int n, float eps) {
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
        const float v = x[j];
        sq[j] = __fmul_rn(v, v);
    }
    __syncthreads();
    __shared__ float inv_rms;
    if (threadIdx.x == 0) {
        float ss = 0.0f;
        int j = 0;
        for (; j + 4 <= n; j += 4) {
            const float4 q = *reinterpret_cast<const float4 *>(sq + j);
            ss = __fadd_rn(ss, q.x);
            ss = __fadd_rn(ss, q.y);
            ss = __fadd_rn(ss, q.z);
            ss = __fadd_rn(ss, q.w);
        }
        for (; j < n; j++) ss = __fadd_rn(ss, sq[j]);
        ss = __fdiv_rn(ss, (float)n);
        ss = __fadd_rn(ss, eps);
        inv_rms = __fdiv_rn(1.0f, __fsqrt_rn(ss));
    }
    __syncthreads();
    const float s = inv_rms;
    for (int j = threadIdx.x; j < n; j += blockDim.x) o[j] = __fmul_rn(w[j], __fmul_rn(s, x[j]));
    __syncthreads();
}

// final rmsnorm + quantize (qwen.c:569-570) into global xq/xs for the head, one CTA
__global__ void __launch_bounds__(kThreads) norm_quant_kernel(const float *x, const float *norm_w, float eps, int n,
                                                              int8_t *xq, float *xs) {
    __shared__ __align__(16) float xb[kMaxDim];
    __shared__ __align__(16) float sq[kMaxDim];
    wait_for_producer();
    rmsnorm_smem(xb, sq, x, norm_w, n, eps);
    for (int g = threadIdx.x; g < n / 32; g += blockDim.x) {
        int8_t q[32];
        xs[g] = quantize_group<32>(xb, g, kXQuantizeQwen, q);
#pragma unroll
        for (int i = 0; i < 32; i++) xq[32 * g + i] = q[i];
    }
    allow_consumer();
}

// ---------------------------------------------------------------------------------------------------------------
// The fused decode matvec: prologue (rmsnorm and/or quantize into shared-memory planes), the group-product stream
// of matvec_kernel over "virtual rows" (rows of up to three matrices), the in-order fold, then an epilogue.
enum Epilogue : int {
    kEpiStore = 0,     // out[row] = v
    kEpiResidual = 1,  // out[row] += v                                    (qwen.c:551, :565)
    kEpiSwiGLU = 2,    // tile = rows of w1 then the same rows of w3; out[row] = silu(g) * u   (qwen.c:558-562)
    kEpiHead = 3,      // out[row] = v, plus the argmax key                 (qwen.c:571, 591-598)
};

struct FusedParams {
    const uint8_t *w[3];
    const uint16_t *ws[3];
    int rows[3];        // rows of each matrix; the output row space is their concatenation (or the pair)
    int n, rt, d;       // columns, output rows per tile, output rows in total
    const float *x;        // fp32 activations to quantize (null: xq/xs given)
    const float *norm_w;   // rmsnorm weight (null: no rmsnorm)
    float eps;
    const int8_t *xq;
    const float *xs;
    float *out;
    State *st;
    ExpTable et;           // the host library's expf (SiLU)
};

template <int BITS, int EPI>
__global__ void __launch_bounds__(kThreads) fused_matvec_kernel(const FusedParams p) {
    constexpr int GB = BITS == 4 ? 16 : 32;
    constexpr int WC = GB / 16;
    constexpr int K = BITS == 4 ? 4 : 2;
    extern __shared__ __align__(16) uint8_t smem[];
    const int n = p.n, ng = n / 32, tid = threadIdx.x;
    const int row0 = blockIdx.x * p.rt;
    const int rows = min(p.rt, p.d - row0);
    const int vrows = EPI == kEpiSwiGLU ? 2 * rows : rows;

    // shared memory: planes | xs | xsum | prod[vrows][ng+1] | row pointers | staging floats for the prologue
    uint4 *xplane = reinterpret_cast<uint4 *>(smem);
    float *xs_s = reinterpret_cast<float *>(xplane + 2 * ng);
    int *xsum_s = reinterpret_cast<int *>(xs_s + ng);
    float *prod = reinterpret_cast<float *>(xsum_s + ng);
    const int vmax = EPI == kEpiSwiGLU ? 2 * p.rt : p.rt;
    const uint8_t **wrow = reinterpret_cast<const uint8_t **>(
        (reinterpret_cast<uintptr_t>(prod + (size_t)vmax * (ng + 1)) + 15) & ~(uintptr_t)15);
    const uint16_t **srow = reinterpret_cast<const uint16_t **>(wrow + vmax);
    float *stage = reinterpret_cast<float *>(srow + vmax);  // 2 * n floats when the prologue normalizes

    // row pointers of this tile (weights are constant: set them up before waiting on the producer)
    for (int vr = tid; vr < vrows; vr += kThreads) {
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
        wrow[vr] = wb + (size_t)r * ng * GB;
        srow[vr] = sb + (size_t)r * ng;
    }
    wait_for_producer();

    // prologue: activations into the planes
    if (p.x) {
        const float *src = p.x;
        if (p.norm_w) {
            rmsnorm_smem(stage, stage + n, p.x, p.norm_w, n, p.eps);
            src = stage;
        }
        for (int g = tid; g < ng; g += kThreads) {
            int8_t q[32];
            xs_s[g] = quantize_group<32>(src, g, kXQuantizeQwen, q);
            uint32_t wv[8];
#pragma unroll
            for (int j = 0; j < 8; j++)
                wv[j] = (uint32_t)(uint8_t)q[4 * j] | (uint32_t)(uint8_t)q[4 * j + 1] << 8 |
                        (uint32_t)(uint8_t)q[4 * j + 2] << 16 | (uint32_t)(uint8_t)q[4 * j + 3] << 24;
            if (BITS == 4) {
                uint32_t *ev = reinterpret_cast<uint32_t *>(&xplane[g]);
                uint32_t *od = reinterpret_cast<uint32_t *>(&xplane[ng + g]);
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    ev[j] = __byte_perm(wv[2 * j], wv[2 * j + 1], 0x6420);
                    od[j] = __byte_perm(wv[2 * j], wv[2 * j + 1], 0x7531);
                }
            } else {
                xplane[g] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
                xplane[ng + g] = make_uint4(wv[4], wv[5], wv[6], wv[7]);
            }
        }
    } else {
        for (int c = tid; c < n / 16; c += kThreads) {
            const uint4 a = *reinterpret_cast<const uint4 *>(p.xq + 16 * c);
            const int g = c >> 1, k = c & 1;
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
        }
        for (int g = tid; g < ng; g += kThreads) xs_s[g] = p.xs[g];
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

    // group products of the tile's virtual rows
    const int units = vrows * ng;
    int r = tid / ng, g = tid % ng;
    const int dr = kThreads / ng, dg = kThreads % ng;
    for (int base = tid; base < units; base += K * kThreads) {
        uint4 wv[K][WC];
        uint32_t hs[K];
        int rr = r, gg = g;
#pragma unroll
        for (int k = 0; k < K; k++) {
            if (base + k * kThreads < units) {
                const uint8_t *src = wrow[rr] + (size_t)gg * GB;
#pragma unroll
                for (int c = 0; c < WC; c++) wv[k][c] = ld_weights(src + 16 * c);
                hs[k] = ld_u16(srow[rr] + gg);
            }
            gg += dg;
            rr += dr;
            if (gg >= ng) { gg -= ng; rr++; }
        }
#pragma unroll
        for (int k = 0; k < K; k++) {
            if (base + k * kThreads < units) {
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
                prod[r * (ng + 1) + g] = __fmul_rn(__fmul_rn(__int2float_rn(acc), scale_from_f16(hs[k])), xs_s[g]);
            }
            g += dg;
            r += dr;
            if (g >= ng) { g -= ng; r++; }
        }
    }
    __syncthreads();
    allow_consumer();

    // in-order fold of each virtual row, then the epilogue
    float v = 0.0f;
    if (tid < vrows) {
        const float *pr = prod + tid * (ng + 1);
#pragma unroll 8
        for (int j = 0; j < ng; j++) v = __fadd_rn(v, pr[j]);
    }
    if (EPI == kEpiStore) {
        if (tid < rows) p.out[row0 + tid] = v;
    } else if (EPI == kEpiResidual) {
        if (tid < rows) p.out[row0 + tid] = __fadd_rn(p.out[row0 + tid], v);
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
        if ((tid & 31) == 0 && tid < ((rows + 31) & ~31) && key) atomicMax(&p.st->key, key);
    }
}

inline size_t fused_smem_bytes(int n, int rt, int epi, bool normalize) {
    const int ng = n / 32;
    const int vmax = epi == kEpiSwiGLU ? 2 * rt : rt;
    size_t b = (size_t)2 * ng * 16 + (size_t)ng * 8 + (size_t)vmax * (ng + 1) * 4;
    b = (b + 15) & ~(size_t)15;
    b += (size_t)vmax * 16;
    if (normalize) b += (size_t)2 * n * 4;
    return b;
}

// ---------------------------------------------------------------------------------------------------------------
// attention for one query head (qwen.c:521-546): biases, NeoX RoPE (pairs i, i + hs/2), the KV-cache write of
// this position, scores q.k / sqrt(hs) in order over the head's elements, softmax in order, weighted values in
// order of position.
struct AttnParams {
    const float *qkv;   // raw outputs of the qkv matvec: q (dim) | k (kv_dim) | v (kv_dim)
    const float *bq, *bk, *bv;
    const float *rope;  // per position: cos[hs/2] then sin[hs/2]
    float *kcache, *vcache;  // this layer's (ctx, kv_dim)
    float *xb;          // dim outputs
    int dim, kv_dim, hs, kv_mul;
    State *st;
    ExpTable et;        // the host library's expf (softmax)
};

__global__ void __launch_bounds__(kThreads) attention_kernel(const AttnParams p) {
    __shared__ __align__(16) float q[kMaxHead], kc[kMaxHead], vc[kMaxHead];
    __shared__ __align__(16) float att[kMaxCtx];
    __shared__ float red[kThreads / 32];
    __shared__ float s_max, s_sum;
    const int h = blockIdx.x, kvh = h / p.kv_mul, hs = p.hs, half = hs / 2, tid = threadIdx.x;
    wait_for_producer();
    const int pos = p.st->pos;
    const float *cs = p.rope + (size_t)pos * hs;
    const float *qr = p.qkv + h * hs, *kr = p.qkv + p.dim + kvh * hs, *vr = p.qkv + p.dim + p.kv_dim + kvh * hs;
    if (tid < half) {
        const float c = cs[tid], s = cs[half + tid];
        float a = __fadd_rn(qr[tid], p.bq[h * hs + tid]), b = __fadd_rn(qr[tid + half], p.bq[h * hs + tid + half]);
        q[tid] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
        q[tid + half] = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
        a = __fadd_rn(kr[tid], p.bk[kvh * hs + tid]);
        b = __fadd_rn(kr[tid + half], p.bk[kvh * hs + tid + half]);
        kc[tid] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
        kc[tid + half] = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
    }
    if (tid < hs) vc[tid] = __fadd_rn(vr[tid], p.bv[kvh * hs + tid]);
    __syncthreads();
    if (h % p.kv_mul == 0 && tid < hs) {  // one writer per kv head
        p.kcache[(size_t)pos * p.kv_dim + kvh * hs + tid] = kc[tid];
        p.vcache[(size_t)pos * p.kv_dim + kvh * hs + tid] = vc[tid];
    }
    // scores
    const float scale = __fsqrt_rn((float)hs);
    for (int t = tid; t <= pos; t += kThreads) {
        const float *kt = t == pos ? kc : p.kcache + (size_t)t * p.kv_dim + kvh * hs;
        float score = 0.0f;
        for (int i = 0; i < hs; i += 4) {
            const float4 k4 = *reinterpret_cast<const float4 *>(kt + i);
            score = __fadd_rn(score, __fmul_rn(q[i], k4.x));
            score = __fadd_rn(score, __fmul_rn(q[i + 1], k4.y));
            score = __fadd_rn(score, __fmul_rn(q[i + 2], k4.z));
            score = __fadd_rn(score, __fmul_rn(q[i + 3], k4.w));
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
    if (tid == 0) {
        float sum = 0.0f;
        for (int t = 0; t <= pos; t++) sum = __fadd_rn(sum, att[t]);
        s_sum = sum;
    }
    __syncthreads();
    const float sum = s_sum;
    for (int t = tid; t <= pos; t += kThreads) att[t] = __fdiv_rn(att[t], sum);
    __syncthreads();
    allow_consumer();
    // weighted values, in order of position
    if (tid < hs) {
        float acc = 0.0f;
        const float *vcol = p.vcache + kvh * hs + tid;
        for (int t = 0; t < pos; t++) acc = __fadd_rn(acc, __fmul_rn(att[t], vcol[(size_t)t * p.kv_dim]));
        acc = __fadd_rn(acc, __fmul_rn(att[pos], vc[tid]));
        p.xb[h * hs + tid] = acc;
    }
}

// next token (qwen.c:674-700): the prompt while it lasts, then the greedy head row's token id
__global__ void next_token_kernel(State *st, const int *prompt, const int32_t *head_ids, int *ids, int cap) {
    wait_for_producer();
    if (threadIdx.x != 0) return;
    const int pos = st->pos;
    const unsigned long long key = st->key;
    // no key: every logit was NaN; the reference's strict `>` then keeps row 0 (qwen.c:591-598)
    const int row = key ? (int)(~(uint32_t)(key & 0xffffffffu)) : 0;
    st->last_row = row;
    if (st->n_prompt >= 0) {
        int next;
        if (pos + 1 < st->n_prompt) {
            next = prompt[pos + 1];
        } else {
            next = head_ids[row];
            if (st->n_gen < cap) ids[st->n_gen] = next;
            st->n_gen++;
        }
        st->token = next;
    }
    st->pos = pos + 1;
}

// ---------------------------------------------------------------------------------------------------------------
struct Config {
    int dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, head_k, max_seq_len, group_size, emb_bits;
    float rope_theta, rms_eps;
};

struct Mat {
    const uint8_t *w;
    const uint16_t *s;
};

struct Model {
    Config c;
    int hs = 0, kv_dim = 0, ctx = 0;
    int device = 0;
    bool pdl = true;
    cudaStream_t stream = nullptr;
    cudaGraphExec_t graph = nullptr;
    uint8_t *image = nullptr;  // the whole .qwb on the device, same byte offsets as the file
    size_t image_bytes = 0;
    const float *attn_norm, *ffn_norm, *bq, *bk, *bv, *out_norm;
    const int32_t *head_ids;
    std::vector<Mat> wq, wk, wv, wo, w1, w2, w3;
    Mat head, emb;
    float *x = nullptr, *xb = nullptr, *qkv = nullptr, *hb = nullptr, *logits = nullptr, *kcache = nullptr,
          *vcache = nullptr, *rope = nullptr, *xs = nullptr;
    int8_t *xq = nullptr;
    int *prompt = nullptr, *ids = nullptr;
    State *st = nullptr;
    int kernels_per_step = 0;
    ExpTable et = {};
    // pinned ring of states for asynchronous rewinds (a slot is reused after kRing rewinds)
    static constexpr int kRing = 256;
    State *ring = nullptr;
    int ring_next = 0;
    // the step again, with an event before every kernel and no programmatic overlap: per-kernel durations
    cudaGraphExec_t prof_graph = nullptr;
    std::vector<cudaEvent_t> prof_ev;
    struct Info { const char *kind; int layer; };
    std::vector<Info> info;  // one per kernel of the step, in launch order
};

// qwen.c:195-199: every array starts on 64 bytes
static size_t take(size_t *off, size_t bytes) {
    const size_t a = *off;
    *off += (bytes + 63) & ~(size_t)63;
    return a;
}

template <typename... KArgs, typename... Args>
static cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
                          Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    if (pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

template <int BITS, int EPI>
static cudaError_t launch_fused(Model &m, FusedParams p, int *count) {
    const bool norm = p.norm_w != nullptr;
    const size_t smem = fused_smem_bytes(p.n, p.rt, EPI, norm);
    (*count)++;
    return launch(fused_matvec_kernel<BITS, EPI>, dim3((p.d + p.rt - 1) / p.rt), dim3(kThreads), smem, m.stream,
                  m.pdl, p);
}

// Enqueues one forward step on m.stream (captured into a graph by the caller). With `ev`, records ev[k] before
// kernel k and ev[count] after the last one; `info` receives each kernel's kind and layer.
static cudaError_t enqueue_step(Model &m, int *count, cudaEvent_t *ev = nullptr,
                                std::vector<Model::Info> *info = nullptr, float *trace = nullptr) {
    const Config &c = m.c;
    cudaError_t e;
    *count = 0;
    // inside stream capture a plain event record is only a dependency marker; External makes it a graph node
    auto mark = [&](const char *kind, int layer) -> cudaError_t {
        if (info) info->push_back(Model::Info{kind, layer});
        return ev ? cudaEventRecordWithFlags(ev[*count], m.stream, cudaEventRecordExternal) : cudaSuccess;
    };
    // with `trace`, x is copied out after each residual update: trace[0] after the embedding, then per layer
    // after attention (2l + 1) and after the FFN (2l + 2)
    auto snap = [&](int slot) -> cudaError_t {
        return trace ? cudaMemcpyAsync(trace + (size_t)slot * c.dim, m.x, c.dim * 4, cudaMemcpyDeviceToDevice,
                                       m.stream)
                     : cudaSuccess;
    };
    if ((e = mark("embed", -1)) != cudaSuccess) return e;
    e = launch(embed_kernel, dim3((c.dim + 255) / 256), dim3(256), 0, m.stream, m.pdl, (const int8_t *)m.emb.w,
               m.emb.s, m.x, c.dim, m.st);
    (*count)++;
    if (e != cudaSuccess || (e = snap(0)) != cudaSuccess) return e;
    const int dim = c.dim, hid = c.hidden_dim, kv = m.kv_dim;
    for (int l = 0; l < c.n_layers; l++) {
        FusedParams p = {};
        // qkv: rmsnorm + quantize + [wq; wk; wv]
        p.w[0] = m.wq[l].w; p.ws[0] = m.wq[l].s; p.rows[0] = dim;
        p.w[1] = m.wk[l].w; p.ws[1] = m.wk[l].s; p.rows[1] = kv;
        p.w[2] = m.wv[l].w; p.ws[2] = m.wv[l].s; p.rows[2] = kv;
        p.n = dim; p.d = dim + 2 * kv; p.rt = 8;
        p.x = m.x; p.norm_w = m.attn_norm + (size_t)l * dim; p.eps = c.rms_eps;
        p.out = m.qkv; p.st = m.st;
        if ((e = mark("qkv", l)) != cudaSuccess || (e = launch_fused<4, kEpiStore>(m, p, count)) != cudaSuccess)
            return e;
        // attention
        AttnParams a;
        a.qkv = m.qkv;
        a.bq = m.bq + (size_t)l * dim; a.bk = m.bk + (size_t)l * kv; a.bv = m.bv + (size_t)l * kv;
        a.rope = m.rope;
        a.kcache = m.kcache + (size_t)l * m.ctx * kv; a.vcache = m.vcache + (size_t)l * m.ctx * kv;
        a.xb = m.xb; a.dim = dim; a.kv_dim = kv; a.hs = m.hs; a.kv_mul = c.n_heads / c.n_kv_heads; a.st = m.st;
        a.et = m.et;
        if ((e = mark("attention", l)) != cudaSuccess) return e;
        if ((e = launch(attention_kernel, dim3(c.n_heads), dim3(kThreads), 0, m.stream, m.pdl, a)) != cudaSuccess)
            return e;
        (*count)++;
        // o: quantize(xb) + wo, x += out
        p = FusedParams{};
        p.w[0] = m.wo[l].w; p.ws[0] = m.wo[l].s; p.rows[0] = dim;
        p.n = dim; p.d = dim; p.rt = 8; p.x = m.xb; p.out = m.x; p.st = m.st;
        if ((e = mark("o_proj", l)) != cudaSuccess || (e = launch_fused<4, kEpiResidual>(m, p, count)) != cudaSuccess ||
            (e = snap(2 * l + 1)) != cudaSuccess)
            return e;
        // gate/up: rmsnorm + quantize + (w1, w3) paired rows, SwiGLU -> hb
        p = FusedParams{};
        p.w[0] = m.w1[l].w; p.ws[0] = m.w1[l].s; p.rows[0] = hid;
        p.w[1] = m.w3[l].w; p.ws[1] = m.w3[l].s; p.rows[1] = hid;
        p.n = dim; p.d = hid; p.rt = 16;
        p.x = m.x; p.norm_w = m.ffn_norm + (size_t)l * dim; p.eps = c.rms_eps;
        p.out = m.hb; p.st = m.st; p.et = m.et;
        if ((e = mark("gate_up", l)) != cudaSuccess || (e = launch_fused<4, kEpiSwiGLU>(m, p, count)) != cudaSuccess)
            return e;
        // down: quantize(hb) + w2, x += out
        p = FusedParams{};
        p.w[0] = m.w2[l].w; p.ws[0] = m.w2[l].s; p.rows[0] = dim;
        p.n = hid; p.d = dim; p.rt = 8; p.x = m.hb; p.out = m.x; p.st = m.st;
        if ((e = mark("down", l)) != cudaSuccess || (e = launch_fused<4, kEpiResidual>(m, p, count)) != cudaSuccess ||
            (e = snap(2 * l + 2)) != cudaSuccess)
            return e;
    }
    // final norm + quantize, head, next token
    if ((e = mark("final_norm", -1)) != cudaSuccess) return e;
    if ((e = launch(norm_quant_kernel, dim3(1), dim3(kThreads), 0, m.stream, m.pdl, m.x, m.out_norm, c.rms_eps, dim,
                    m.xq, m.xs)) != cudaSuccess)
        return e;
    (*count)++;
    FusedParams p = {};
    p.w[0] = m.head.w; p.ws[0] = m.head.s; p.rows[0] = c.head_k;
    p.n = dim; p.d = c.head_k; p.rt = 32; p.xq = m.xq; p.xs = m.xs; p.out = m.logits; p.st = m.st;
    if ((e = mark("head", -1)) != cudaSuccess || (e = launch_fused<8, kEpiHead>(m, p, count)) != cudaSuccess)
        return e;
    if ((e = mark("next_token", -1)) != cudaSuccess) return e;
    e = launch(next_token_kernel, dim3(1), dim3(32), 0, m.stream, m.pdl, m.st, (const int *)m.prompt, m.head_ids,
               m.ids, m.ctx);
    (*count)++;
    if (e == cudaSuccess && ev) e = cudaEventRecordWithFlags(ev[*count], m.stream, cudaEventRecordExternal);
    return e;
}

// Algorithmic bytes of kernel k of the step at position `pos`: every byte the kernel must move at least once
// (weights and scales, activations in and out, norm weights, KV-cache rows read and written).
static double kernel_bytes(const Model &m, int k, int pos) {
    const Config &c = m.c;
    const double dim = c.dim, hid = c.hidden_dim, kv = m.kv_dim, ng = dim / 32, ngh = hid / 32;
    const char *kind = m.info[k].kind;
    auto q4 = [](double d, double n) { return d * n / 2 + d * (n / 32) * 2; };
    if (!strcmp(kind, "embed")) return dim + ng * 2 + dim * 4;
    if (!strcmp(kind, "qkv")) return q4(dim + 2 * kv, dim) + dim * 4 * 2 + (dim + 2 * kv) * 4;
    if (!strcmp(kind, "attention"))
        return (dim + 2 * kv) * 4 * 2 + m.hs * 4 + 2.0 * pos * kv * 4 + 2 * kv * 4 + dim * 4;
    if (!strcmp(kind, "o_proj")) return q4(dim, dim) + dim * 4 + dim * 8;
    if (!strcmp(kind, "gate_up")) return 2 * q4(hid, dim) + dim * 4 * 2 + hid * 4;
    if (!strcmp(kind, "down")) return q4(dim, hid) + hid * 4 + dim * 8;
    if (!strcmp(kind, "final_norm")) return dim * 4 * 2 + dim + ng * 4;
    if (!strcmp(kind, "head")) return (double)c.head_k * dim + (double)c.head_k * ng * 2 + dim + ng * 4 + c.head_k * 4.0;
    (void)ngh;
    return 16;
}

static void destroy(Model *m) {
    if (!m) return;
    if (m->stream) cudaStreamSynchronize(m->stream);
    if (m->graph) cudaGraphExecDestroy(m->graph);
    if (m->prof_graph) cudaGraphExecDestroy(m->prof_graph);
    for (cudaEvent_t e : m->prof_ev) cudaEventDestroy(e);
    if (m->ring) cudaFreeHost(m->ring);
    void *bufs[] = {m->image, m->x, m->xb, m->qkv, m->hb, m->logits, m->kcache, m->vcache, m->rope, m->xs, m->xq,
                    m->prompt, m->ids, m->st};
    for (void *b : bufs)
        if (b) cudaFree(b);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
}

static double now_s() {
    timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return t.tv_sec + t.tv_nsec * 1e-9;
}

static double timeout_s() {
    const char *e = getenv("MATVEC_TIMEOUT_S");
    const double v = e ? atof(e) : 5.0;
    return v > 0 ? v : 5.0;
}

// Polls the stream against a deadline instead of blocking forever (the reference gives up after 5 s).
static int wait_stream(Model &m, const char *who, double budget_s) {
    const double deadline = now_s() + budget_s;
    for (unsigned i = 1;; i++) {
        const cudaError_t e = cudaStreamQuery(m.stream);
        if (e == cudaSuccess) return 0;
        if (e != cudaErrorNotReady) {
            set_error("%s: device error: %s", who, cudaGetErrorString(e));
            return -1;
        }
        if (i % 256 == 0 && now_s() > deadline) {
            set_error("%s: the device did not finish in %.1f s", who, budget_s);
            return -1;
        }
    }
}

}  // namespace qwen
}  // namespace mvb

using namespace mvb;
using namespace mvb::qwen;

extern "C" void *mvb_qwen_load(const void *image, size_t bytes, int ctx) {
    clear_error();
    if (!image || bytes < 256) {
        set_error("mvb_qwen_load: no .qwb image");
        return nullptr;
    }
    const uint8_t *b = static_cast<const uint8_t *>(image);
    uint32_t version;
    memcpy(&version, b + 4, 4);
    if (memcmp(b, "QWB1", 4) || version != 1) {
        set_error("mvb_qwen_load: not a .qwb version 1 image");
        return nullptr;
    }
    Model *m = new Model;
    memcpy(&m->c, b + 8, sizeof(Config));
    Config &c = m->c;
    // qwen.c:223-228's checks, plus this implementation's own limits
    if (c.group_size != 32 || c.emb_bits != 8 || c.n_heads <= 0 || c.n_kv_heads <= 0 || c.dim % c.n_heads ||
        c.n_heads % c.n_kv_heads || (c.dim / c.n_heads) % 2 || c.dim % 128 || c.hidden_dim % 128 ||
        (c.dim / c.n_heads * c.n_kv_heads) % 16 || c.dim > kMaxDim || c.hidden_dim > kMaxN || c.dim / c.n_heads > kMaxHead ||
        (c.dim / c.n_heads) % 4 || c.head_k <= 0 || c.vocab_size <= 0 || c.n_layers <= 0) {
        set_error("mvb_qwen_load: unsupported config (group %d, embedding %d-bit, dim %d, hidden %d, heads %d/%d)",
                  c.group_size, c.emb_bits, c.dim, c.hidden_dim, c.n_heads, c.n_kv_heads);
        delete m;
        return nullptr;
    }
    m->hs = c.dim / c.n_heads;
    m->kv_dim = m->hs * c.n_kv_heads;
    m->ctx = ctx < c.max_seq_len ? ctx : c.max_seq_len;  // qwen.c:325
    if (m->ctx < 2 || m->ctx > kMaxCtx) {
        set_error("mvb_qwen_load: context %d outside [2, %d]", m->ctx, kMaxCtx);
        delete m;
        return nullptr;
    }
    // walk the file like qwen.c:237-262
    const int L = c.n_layers, dim = c.dim, kv = m->kv_dim, hid = c.hidden_dim;
    size_t off = 256;
    const size_t o_attn = take(&off, (size_t)L * dim * 4), o_ffn = take(&off, (size_t)L * dim * 4),
                 o_bq = take(&off, (size_t)L * dim * 4), o_bk = take(&off, (size_t)L * kv * 4),
                 o_bv = take(&off, (size_t)L * kv * 4), o_norm = take(&off, (size_t)dim * 4),
                 o_ids = take(&off, (size_t)c.head_k * 4);
    struct MatOff { size_t w, s; };
    auto mats = [&](int count, int d, int n, int bits) {
        std::vector<MatOff> v(count);
        for (auto &x : v) {
            x.w = take(&off, (size_t)d * n * bits / 8);
            x.s = take(&off, (size_t)d * n / 32 * 2);
        }
        return v;
    };
    auto q = mats(L, dim, dim, 4), k = mats(L, kv, dim, 4), vv = mats(L, kv, dim, 4), o = mats(L, dim, dim, 4),
         g = mats(L, hid, dim, 4), dn = mats(L, dim, hid, 4), u = mats(L, hid, dim, 4);
    auto hd = mats(1, c.head_k, dim, 8), em = mats(1, c.vocab_size, dim, 8);
    if (off != bytes) {
        set_error("mvb_qwen_load: image is %zu bytes, but the header describes %zu", bytes, off);
        delete m;
        return nullptr;
    }
    const int32_t *ids = reinterpret_cast<const int32_t *>(b + o_ids);
    for (int i = 0; i < c.head_k; i++)
        if (ids[i] < 0 || ids[i] >= c.vocab_size) {
            set_error("mvb_qwen_load: head_ids[%d] = %d outside the vocabulary", i, ids[i]);
            delete m;
            return nullptr;
        }
    cudaError_t e = cudaGetDevice(&m->device);
    if (const char *pd = getenv("MVB_PDL")) m->pdl = atoi(pd) != 0;
    auto fail = [&](const char *what) -> void * {
        set_error("mvb_qwen_load: %s: %s", what, cudaGetErrorString(e));
        destroy(m);
        return nullptr;
    };
    if (e != cudaSuccess) return fail("no device");
    if ((e = cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking)) != cudaSuccess) return fail("stream");
    if ((e = cudaMalloc(&m->image, bytes)) != cudaSuccess) return fail("weights");
    if ((e = cudaMemcpy(m->image, image, bytes, cudaMemcpyHostToDevice)) != cudaSuccess) return fail("upload");
    m->image_bytes = bytes;
    auto at = [&](size_t o) { return m->image + o; };
    m->attn_norm = (const float *)at(o_attn); m->ffn_norm = (const float *)at(o_ffn);
    m->bq = (const float *)at(o_bq); m->bk = (const float *)at(o_bk); m->bv = (const float *)at(o_bv);
    m->out_norm = (const float *)at(o_norm); m->head_ids = (const int32_t *)at(o_ids);
    auto conv = [&](const std::vector<MatOff> &v, std::vector<Mat> &dst) {
        for (auto &x : v) dst.push_back(Mat{at(x.w), (const uint16_t *)at(x.s)});
    };
    conv(q, m->wq); conv(k, m->wk); conv(vv, m->wv); conv(o, m->wo); conv(g, m->w1); conv(dn, m->w2); conv(u, m->w3);
    m->head = Mat{at(hd[0].w), (const uint16_t *)at(hd[0].s)};
    m->emb = Mat{at(em[0].w), (const uint16_t *)at(em[0].s)};
    // RoPE table, exactly qwen.c:504-508 per position
    std::vector<float> rope((size_t)m->ctx * m->hs);
    for (int pos = 0; pos < m->ctx; pos++)
        for (int i = 0; i < m->hs / 2; i++) {
            double a = pos * pow(c.rope_theta, -2.0 * i / m->hs);
            rope[(size_t)pos * m->hs + i] = (float)cos(a);
            rope[(size_t)pos * m->hs + m->hs / 2 + i] = (float)sin(a);
        }
    const size_t kvbytes = (size_t)L * m->ctx * kv * 4;
    if ((e = cudaMalloc(&m->x, dim * 4)) != cudaSuccess || (e = cudaMalloc(&m->xb, dim * 4)) != cudaSuccess ||
        (e = cudaMalloc(&m->qkv, (dim + 2 * kv) * 4)) != cudaSuccess ||
        (e = cudaMalloc(&m->hb, (size_t)hid * 4)) != cudaSuccess ||
        (e = cudaMalloc(&m->logits, (size_t)c.head_k * 4)) != cudaSuccess ||
        (e = cudaMalloc(&m->kcache, kvbytes)) != cudaSuccess || (e = cudaMalloc(&m->vcache, kvbytes)) != cudaSuccess ||
        (e = cudaMalloc(&m->rope, rope.size() * 4)) != cudaSuccess ||
        (e = cudaMalloc(&m->xq, dim)) != cudaSuccess || (e = cudaMalloc(&m->xs, dim / 32 * 4)) != cudaSuccess ||
        (e = cudaMalloc(&m->prompt, (size_t)m->ctx * 4)) != cudaSuccess ||
        (e = cudaMalloc(&m->ids, (size_t)m->ctx * 4)) != cudaSuccess ||
        (e = cudaMalloc(&m->st, sizeof(State))) != cudaSuccess)
        return fail("buffers");
    if ((e = cudaMemcpy(m->rope, rope.data(), rope.size() * 4, cudaMemcpyHostToDevice)) != cudaSuccess ||
        (e = cudaMemset(m->kcache, 0, kvbytes)) != cudaSuccess || (e = cudaMemset(m->vcache, 0, kvbytes)) != cudaSuccess ||
        (e = cudaMemset(m->st, 0, sizeof(State))) != cudaSuccess)
        return fail("init");
    if ((e = cudaHostAlloc(&m->ring, sizeof(State) * Model::kRing, cudaHostAllocDefault)) != cudaSuccess)
        return fail("pinned state");
    m->et = expf_table_device();
    if (!m->et.slots) {
        e = cudaErrorUnknown;
        return fail("expf table");
    }
    // capture one forward step, then the instrumented copy (events between kernels, no programmatic overlap)
    for (int pass = 0; pass < 2; pass++) {
        cudaGraph_t graph;
        int count = 0;
        const bool pdl = m->pdl;
        if (pass == 1) {
            m->pdl = false;
            m->prof_ev.resize(m->kernels_per_step + 1);
            for (auto &ev : m->prof_ev)
                if ((e = cudaEventCreate(&ev)) != cudaSuccess) return fail("events");
        }
        if ((e = cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal)) != cudaSuccess)
            return fail("capture");
        cudaError_t le = pass == 0 ? enqueue_step(*m, &count, nullptr, &m->info)
                                   : enqueue_step(*m, &count, m->prof_ev.data(), nullptr);
        e = cudaStreamEndCapture(m->stream, &graph);
        m->pdl = pdl;
        if (le != cudaSuccess) {
            e = le;
            return fail("kernel launch");
        }
        if (e != cudaSuccess) return fail("capture");
        e = cudaGraphInstantiate(pass == 0 ? &m->graph : &m->prof_graph, graph, 0);
        cudaGraphDestroy(graph);
        if (e != cudaSuccess) return fail("graph");
        if (pass == 0) m->kernels_per_step = count;
    }
    return m;
}

extern "C" void mvb_qwen_free(void *model) { destroy(static_cast<Model *>(model)); }

extern "C" int mvb_qwen_config(void *model, int *out) {
    Model *m = static_cast<Model *>(model);
    if (!m || !out) return -1;
    const Config &c = m->c;
    const int v[] = {c.dim, c.hidden_dim, c.n_layers, c.n_heads, c.n_kv_heads, c.vocab_size, c.head_k, m->ctx,
                     m->kernels_per_step};
    memcpy(out, v, sizeof v);
    return 0;
}

extern "C" void *mvb_qwen_stream(void *model) { return model ? static_cast<Model *>(model)->stream : nullptr; }

static int set_state(Model &m, int token, int pos, int n_prompt) {
    State s = {};
    s.token = token;
    s.pos = pos;
    s.n_prompt = n_prompt;
    const cudaError_t e = cudaMemcpyAsync(m.st, &s, sizeof s, cudaMemcpyHostToDevice, m.stream);
    if (e != cudaSuccess) {
        set_error("mvb_qwen: %s", cudaGetErrorString(e));
        return -1;
    }
    return wait_stream(m, "mvb_qwen", timeout_s());  // s lives on this stack frame
}

// Launches the captured step `count` times on the model's stream (asynchronous).
extern "C" int mvb_qwen_launch(void *model, int count) {
    Model *m = static_cast<Model *>(model);
    if (!m || count < 0) return -1;
    for (int i = 0; i < count; i++) {
        const cudaError_t e = cudaGraphLaunch(m->graph, m->stream);
        if (e != cudaSuccess) {
            set_error("mvb_qwen_launch: %s", cudaGetErrorString(e));
            return -1;
        }
    }
    return 0;
}

extern "C" int mvb_qwen_forward(void *model, int token, int pos, float *logits) {
    Model *m = static_cast<Model *>(model);
    if (!m) return -1;
    if (pos < 0 || pos >= m->ctx || token < 0 || token >= m->c.vocab_size) {
        set_error("mvb_qwen_forward: token %d / position %d out of range", token, pos);
        return -1;
    }
    if (set_state(*m, token, pos, -1) || mvb_qwen_launch(m, 1)) return -1;
    if (logits && cudaMemcpyAsync(logits, m->logits, (size_t)m->c.head_k * 4, cudaMemcpyDeviceToHost, m->stream) !=
                      cudaSuccess) {
        set_error("mvb_qwen_forward: logits download failed");
        return -1;
    }
    if (wait_stream(*m, "mvb_qwen_forward", timeout_s())) return -1;
    State &s = m->ring[m->ring_next];
    m->ring_next = (m->ring_next + 1) % Model::kRing;
    if (cudaMemcpyAsync(&s, m->st, sizeof s, cudaMemcpyDeviceToHost, m->stream) != cudaSuccess ||
        wait_stream(*m, "mvb_qwen_forward", timeout_s()))
        return -1;
    return s.last_row;
}

// Feeds prompt[0 .. n-2] (positions 0 .. n-2), leaving prompt[n-1] as the token of position n-1: the state
// qwen.c's generate() is in just before its first sampled token.
extern "C" int mvb_qwen_prefill(void *model, const int *prompt, int n) {
    Model *m = static_cast<Model *>(model);
    if (!m || !prompt || n < 1 || n >= m->ctx) {
        set_error("mvb_qwen_prefill: need 1 <= n < ctx");
        return -1;
    }
    for (int i = 0; i < n; i++)
        if (prompt[i] < 0 || prompt[i] >= m->c.vocab_size) {
            set_error("mvb_qwen_prefill: token id %d out of range", prompt[i]);
            return -1;
        }
    if (cudaMemcpyAsync(m->prompt, prompt, (size_t)n * 4, cudaMemcpyHostToDevice, m->stream) != cudaSuccess) {
        set_error("mvb_qwen_prefill: prompt upload failed");
        return -1;
    }
    if (set_state(*m, prompt[0], 0, n) || mvb_qwen_launch(m, n - 1)) return -1;
    return wait_stream(*m, "mvb_qwen_prefill", timeout_s() + 0.01 * n);
}

// Greedy decode of `steps` tokens from the current state; ids (host) receives them. Returns the count.
extern "C" int mvb_qwen_decode(void *model, int steps, int *ids) {
    Model *m = static_cast<Model *>(model);
    if (!m || steps < 0 || !ids) return -1;
    // read the state behind any rewind still queued on the stream
    State &s = m->ring[m->ring_next];
    m->ring_next = (m->ring_next + 1) % Model::kRing;
    if (cudaMemcpyAsync(&s, m->st, sizeof s, cudaMemcpyDeviceToHost, m->stream) != cudaSuccess) {
        set_error("mvb_qwen_decode: state read failed");
        return -1;
    }
    if (wait_stream(*m, "mvb_qwen_decode", timeout_s())) return -1;
    if (s.n_prompt < 0 || s.pos + steps > m->ctx) {
        set_error("mvb_qwen_decode: no prompt fed, or %d steps from position %d exceed the context %d", steps,
                  s.pos, m->ctx);
        return -1;
    }
    const int first = s.n_gen;
    if (mvb_qwen_launch(m, steps)) return -1;
    if (cudaMemcpyAsync(ids, m->ids + first, (size_t)steps * 4, cudaMemcpyDeviceToHost, m->stream) != cudaSuccess) {
        set_error("mvb_qwen_decode: ids download failed");
        return -1;
    }
    if (wait_stream(*m, "mvb_qwen_decode", timeout_s() + 0.01 * steps)) return -1;
    return steps;
}

// Sets input `token` at position `pos` for the next step (positions below keep their KV cache), asynchronously:
// the state goes up from a pinned ring slot on the model's stream, so a benchmark can enqueue rewind + decode
// steps without host synchronization. A slot is rewritten only kRing rewinds later.
extern "C" int mvb_qwen_rewind(void *model, int token, int pos, int n_prompt) {
    Model *m = static_cast<Model *>(model);
    if (!m || pos < 0 || pos >= m->ctx || token < 0 || token >= m->c.vocab_size) {
        set_error("mvb_qwen_rewind: token %d / position %d out of range", token, pos);
        return -1;
    }
    State &s = m->ring[m->ring_next];
    m->ring_next = (m->ring_next + 1) % Model::kRing;
    s = State{};
    s.token = token;
    s.pos = pos;
    s.n_prompt = n_prompt;
    const cudaError_t e = cudaMemcpyAsync(m->st, &s, sizeof s, cudaMemcpyHostToDevice, m->stream);
    if (e != cudaSuccess) {
        set_error("mvb_qwen_rewind: %s", cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

// Runs the instrumented step once from the current state (which it advances like a normal step) and writes
// each kernel's duration in milliseconds to ms[0 .. count-1]. Returns the kernel count, or -1.
extern "C" int mvb_qwen_profile(void *model, float *ms, int cap) {
    Model *m = static_cast<Model *>(model);
    if (!m || !ms || cap < m->kernels_per_step) return -1;
    cudaError_t e = cudaGraphLaunch(m->prof_graph, m->stream);
    if (e != cudaSuccess) {
        set_error("mvb_qwen_profile: %s", cudaGetErrorString(e));
        return -1;
    }
    if (wait_stream(*m, "mvb_qwen_profile", timeout_s())) return -1;
    for (int k = 0; k < m->kernels_per_step; k++) {
        if ((e = cudaEventElapsedTime(&ms[k], m->prof_ev[k], m->prof_ev[k + 1])) != cudaSuccess) {
            set_error("mvb_qwen_profile: %s", cudaGetErrorString(e));
            return -1;
        }
    }
    return m->kernels_per_step;
}

// One forward at (token, pos) launched directly (not from the graph), copying the residual stream x to `trace`
// (host, (2 * n_layers + 1) * dim floats) after the embedding and after every attention and FFN block.
extern "C" int mvb_qwen_trace(void *model, int token, int pos, float *trace) {
    Model *m = static_cast<Model *>(model);
    if (!m || !trace || pos < 0 || pos >= m->ctx || token < 0 || token >= m->c.vocab_size) {
        set_error("mvb_qwen_trace: bad arguments");
        return -1;
    }
    const size_t n = (size_t)(2 * m->c.n_layers + 1) * m->c.dim;
    float *dev = nullptr;
    int count = 0;
    cudaError_t e = cudaMalloc(&dev, n * 4);
    if (e == cudaSuccess && set_state(*m, token, pos, -1) == 0) {
        e = enqueue_step(*m, &count, nullptr, nullptr, dev);
        if (e == cudaSuccess) e = cudaMemcpyAsync(trace, dev, n * 4, cudaMemcpyDeviceToHost, m->stream);
        if (e == cudaSuccess && wait_stream(*m, "mvb_qwen_trace", timeout_s())) e = cudaErrorUnknown;
    }
    if (dev) cudaFree(dev);
    if (e != cudaSuccess) {
        set_error("mvb_qwen_trace: %s", cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

// Kind ("embed", "qkv", "attention", "o_proj", "gate_up", "down", "final_norm", "head", "next_token"), layer
// (-1 outside the layers) and algorithmic bytes at position `pos` of kernel k of the step. 0, or -1.
extern "C" int mvb_qwen_kernel_info(void *model, int k, int pos, char *kind, int kind_len, int *layer,
                                    double *bytes) {
    Model *m = static_cast<Model *>(model);
    if (!m || k < 0 || k >= (int)m->info.size()) return -1;
    if (kind && kind_len > 0) snprintf(kind, kind_len, "%s", m->info[k].kind);
    if (layer) *layer = m->info[k].layer;
    if (bytes) *bytes = kernel_bytes(*m, k, pos);
    return 0;
}

// qwen.c generate() at temperature 0 (qwen.c:669-712): prompt fed one position at a time, then greedy tokens
// until `steps` are generated, <|im_end|>/<|endoftext|> is sampled, or the context is full. Returns the count.
extern "C" int mvb_qwen_generate(void *model, const int *prompt, int n_prompt, int steps, int *ids) {
    Model *m = static_cast<Model *>(model);
    if (!m || !ids || steps < 1) {
        set_error("mvb_qwen_generate: bad arguments");
        return -1;
    }
    if (mvb_qwen_prefill(model, prompt, n_prompt)) return -1;
    const int room = m->ctx - (n_prompt - 1);
    const int n = steps < room ? steps : room;
    if (mvb_qwen_decode(model, n, ids) != n) return -1;
    for (int i = 0; i < n; i++)
        if (ids[i] == kImEnd || ids[i] == kEndOfText) return i;
    return n;
}

// ---------------------------------------------------------------------------------------------------------------
// The decode's head path without any device allocation: final rmsnorm + quantize (norm_quant_kernel) into a
// scratch that lives in a file-scope device array, then the head matvec reading it. For callers that cannot
// allocate device memory (see mvb_norm_matvec4_static in include/matvec_b200.h).
namespace mvb {
namespace qwen {

constexpr int kStaticNormMatvecMaxN = kMaxDim;  // 2048 columns
// n int8 quantized activations at offset 0, their n/32 fp32 scales at offset kStaticNormMatvecMaxN
static __device__ __align__(256) uint8_t g_norm_matvec_scratch[kStaticNormMatvecMaxN + kStaticNormMatvecMaxN / 32 * 4];

static std::mutex g_scratch_mu;
static std::map<int, uint8_t *> g_scratch_addr;  // device ordinal -> device address of the array

// The array's device address on the current device, looked up once per device. Host code only has a stand-in
// for the array's name; handing that to a kernel would read the wrong memory.
static uint8_t *scratch_address(int dev) {
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    auto it = g_scratch_addr.find(dev);
    if (it != g_scratch_addr.end()) return it->second;
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_norm_matvec_scratch);
    if (e != cudaSuccess || !p) {
        set_error("mvb_norm_matvec4_static: cannot get the scratch address on device %d: %s", dev,
                  cudaGetErrorString(e));
        return nullptr;
    }
    g_scratch_addr[dev] = static_cast<uint8_t *>(p);
    return static_cast<uint8_t *>(p);
}

}  // namespace qwen
}  // namespace mvb

extern "C" int mvb_norm_matvec4_static(const float *x, const float *norm_w, float eps, const void *w, const void *ws,
                                       float *out, int n, int d, int wbits, void *stream) {
    using namespace mvb::qwen;
    if (!x || !norm_w) {
        set_error("mvb_norm_matvec4_static: null pointer argument");
        return -1;
    }
    if (wbits != 4 && wbits != 8) {
        set_error("mvb_norm_matvec4_static: unsupported wbits=%d (need 4 or 8)", wbits);
        return -1;
    }
    if (n <= 0 || n % 32 || n > kStaticNormMatvecMaxN || d <= 0) {
        set_error("mvb_norm_matvec4_static: unsupported n=%d d=%d: this entry point keeps its scratch in a fixed "
                  "device array and takes at most n = %d columns (n %% 32 == 0, d >= 1)", n, d, kStaticNormMatvecMaxN);
        return -1;
    }
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        set_error("mvb_norm_matvec4_static: %s", cudaGetErrorString(e));
        return -1;
    }
    uint8_t *scratch = scratch_address(dev);
    if (!scratch) return -1;
    int8_t *xq = reinterpret_cast<int8_t *>(scratch);
    float *xs = reinterpret_cast<float *>(scratch + kStaticNormMatvecMaxN);
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    norm_quant_kernel<<<1, kThreads, 0, s>>>(x, norm_w, eps, n, xq, xs);
    if ((e = cudaGetLastError()) != cudaSuccess) {
        set_error("mvb_norm_matvec4_static: launch failed: %s", cudaGetErrorString(e));
        return -1;
    }
    return launch_matvec("mvb_norm_matvec4_static", wbits == 4 ? kQ4F16 : kQ8F16, 32, w, ws, xq, xs, nullptr, out, n,
                         d, kXQuantized, s);
}
