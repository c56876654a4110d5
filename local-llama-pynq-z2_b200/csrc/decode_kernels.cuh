// Kernels of the device-resident decode step (qwen_decode.cu). Every kernel:
//   1. loads what does not depend on the previous kernel (its weight tile into registers, norm weights; for the
//      attention the cached keys and values of earlier positions) before it waits for the previous kernel
//      (griddepcontrol.wait), so with programmatic dependent launch these loads overlap the previous kernel;
//   2. turns the previous kernel's fp32 output into this kernel's int8 input in every CTA at once (rmsnorm +
//      quantize, or quantize), reading it with L2 loads;
//   3. computes, letting the next kernel launch (griddepcontrol.launch_dependents) where measurement put it:
//      for most matvecs just before the fold, for qkv at the top (its consumer, the attention, prefetches the
//      KV cache), for the attention after its value sums (Qwen) or before them (runq). Two kernels also have a
//      tail run by their last CTA to finish (an atomic counter that this CTA resets for the next step): the
//      last layer's down projection normalizes x once for the head, and the head picks the next token.
// The kernels serve two model families, chosen by the template parameter FAM:
//   kQwen  qwen.c (qwen/qwen.c): int4/int8 weights with fp16 scales, activations quantized by the reciprocal of
//          the scale, q/k/v biases, NeoX RoPE (pairs i, i + hs/2), a head mapped through head_ids;
//   kRunq  runq.c (runq/runq.c): int8 weights with fp32 scales, activations quantized by dividing by the scale,
//          no biases, interleaved RoPE (pairs 2i, 2i + 1), the classifier's row is the token.
// The arithmetic of every step is the family's reference, operation by operation (see qwen_decode.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "expf_ref.h"
#include "matvec_kernels.cuh"

namespace mvb {
namespace decode {

// model families; the values are the matching activation-quantization modes of matvec_kernels.cuh
constexpr int kQwen = kXQuantizeQwen, kRunq = kXQuantizeRunq;

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

// Timing of the step as the graph runs it (only in the model's stamped copy of the step; null elsewhere): stamp[0]
// keeps ~t of the earliest moment a CTA of the kernel got past its wait for the previous kernel, stamp[1] the
// latest moment a CTA finished, both as atomic maxima of %globaltimer so that zeroed slots need no other setup.
__device__ __forceinline__ void stamp_start(unsigned long long *stamp) {
    if (stamp && threadIdx.x == 0) atomicMax(stamp, ~global_ns());
}
__device__ __forceinline__ void stamp_end(unsigned long long *stamp) {
    if (stamp && threadIdx.x == 0) atomicMax(stamp + 1, global_ns());
}

// Quantizes a long v[0 .. n-1] (more groups of 32 than one pass of quantize_to_planes covers) into the same
// planes: four threads per group, eight consecutive elements each, and two groups per thread at a time, so the
// 152 groups of a 4,864-wide input take two passes instead of five. Same arithmetic as quantize_to_planes (and the
// same group sums into xsum for int4 weights).
template <int BITS, int FAM>
__device__ __forceinline__ void quantize_to_planes_wide(const float *v, int n, uint8_t *planes, float *xs,
                                                        int *xsum) {
    constexpr int kPass = kThreads / 4;  // groups per pass and per slot
    const int ng = n / 32, l = threadIdx.x & 3;
    for (int base = 0; base < ng; base += 2 * kPass) {  // the same trip count in every thread (shuffles)
        float4 f[2][2];
        unsigned m[2];
        int g[2];
#pragma unroll
        for (int h = 0; h < 2; h++) {
            g[h] = base + h * kPass + (threadIdx.x >> 2);
            const bool on = g[h] < ng;
            const float4 *src = reinterpret_cast<const float4 *>(v + 32 * g[h] + 8 * l);
            f[h][0] = on ? src[0] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            f[h][1] = on ? src[1] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            auto bits = [](float x) {
                const float a = fabsf(x);
                return a == a ? __float_as_uint(a) : 0u;
            };
            m[h] = max(max(max(bits(f[h][0].x), bits(f[h][0].y)), max(bits(f[h][0].z), bits(f[h][0].w))),
                       max(max(bits(f[h][1].x), bits(f[h][1].y)), max(bits(f[h][1].z), bits(f[h][1].w))));
        }
#pragma unroll
        for (int h = 0; h < 2; h++) {
            m[h] = max(m[h], __shfl_xor_sync(0xffffffffu, m[h], 1));
            m[h] = max(m[h], __shfl_xor_sync(0xffffffffu, m[h], 2));
        }
        int sum[2] = {0, 0};
#pragma unroll
        for (int h = 0; h < 2; h++) {
            if (g[h] >= ng) continue;
            const float e[8] = {f[h][0].x, f[h][0].y, f[h][0].z, f[h][0].w, f[h][1].x, f[h][1].y, f[h][1].z,
                                f[h][1].w};
            uint32_t q[8];
            float scale;
            if (FAM == kRunq) {  // runq.c: scale = wmax / 127, q = round(x / scale), no guard for a zero scale
                scale = __fdiv_rn(__uint_as_float(m[h]), 127.0f);
#pragma unroll
                for (int i = 0; i < 8; i++) q[i] = (uint8_t)to_int8_x86(roundf(__fdiv_rn(e[i], scale)));
            } else {
                scale = __fmul_rn(__uint_as_float(m[h]), 1.0f / 127.0f);
                const float inv = scale > 0.0f ? __frcp_rn(scale) : 0.0f;  // qwen.c's 1.0f / scale, same value
#pragma unroll
                for (int i = 0; i < 8; i++) q[i] = (uint8_t)to_int8_x86(roundf(__fmul_rn(e[i], inv)));
            }
            if (BITS == 4) {
#pragma unroll
                for (int i = 0; i < 8; i++) sum[h] += (int)(int8_t)q[i];
                // elements 8l + 2i are even-plane bytes 4l + i; elements 8l + 2i + 1 odd-plane bytes 4l + i
                *reinterpret_cast<uint32_t *>(planes + g[h] * 16 + 4 * l) = q[0] | q[2] << 8 | q[4] << 16 | q[6] << 24;
                *reinterpret_cast<uint32_t *>(planes + (ng + g[h]) * 16 + 4 * l) =
                    q[1] | q[3] << 8 | q[5] << 16 | q[7] << 24;
            } else {
                // elements 8l .. 8l+7 are bytes 8(l & 1) .. of chunk l >> 1
                *reinterpret_cast<uint2 *>(planes + ((l >> 1) * ng + g[h]) * 16 + 8 * (l & 1)) =
                    make_uint2(q[0] | q[1] << 8 | q[2] << 16 | q[3] << 24, q[4] | q[5] << 8 | q[6] << 16 | q[7] << 24);
            }
            if (l == 0) xs[g[h]] = scale;
        }
        if (BITS == 4) {  // the groups' sums across their four threads (every thread takes part in the shuffles)
#pragma unroll
            for (int h = 0; h < 2; h++) {
                sum[h] += __shfl_xor_sync(0xffffffffu, sum[h], 1);
                sum[h] += __shfl_xor_sync(0xffffffffu, sum[h], 2);
                if (l == 0 && g[h] < ng) xsum[g[h]] = sum[h];
            }
        }
    }
}

// The rmsnorm weights quantize_to_planes<..., NORM = true> applies in this thread: pass k's four elements of
// group k * kThreads / (GS / 4) + threadIdx.x / (GS / 4). Read before the kernel waits for its producer.
template <int GS>
__device__ __forceinline__ void norm_weights_for_planes(const float *norm_w, int n, float4 (&nw4)[kNormPasses]) {
    constexpr int TPG = GS / 4;
    const int ng = n / GS, l = threadIdx.x % TPG;
#pragma unroll
    for (int k = 0; k < kNormPasses; k++) {
        const int g = k * (kThreads / TPG) + threadIdx.x / TPG;
        nw4[k] = g < ng ? __ldg(reinterpret_cast<const float4 *>(norm_w + GS * g) + l) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

// Quantizes v[0 .. n-1] (shared memory) per group of GS like qwen.c:355-364 (FAM kQwen) or runq.c:244-270
// (kRunq) into xq/xs (global); whole CTA.
template <int FAM, int GS>
__device__ __forceinline__ void quantize_to_global(const float *v, int n, int8_t *xq, float *xs) {
    for (int g = threadIdx.x; g < n / GS; g += blockDim.x) {
        uint32_t q4[GS / 4];
        xs[g] = quantize_group<GS>(v, g, FAM, q4);
        uint4 *dst = reinterpret_cast<uint4 *>(xq + GS * g);
#pragma unroll
        for (int c = 0; c < GS / 16; c++) dst[c] = make_uint4(q4[4 * c], q4[4 * c + 1], q4[4 * c + 2], q4[4 * c + 3]);
    }
}

// rmsnorm (qwen.c:337-344; runq.c:394-407 is the same sequence) of xv (shared memory, n floats) with weight w,
// then quantize per group of GS into xq/xs; whole CTA. xb is n floats of shared scratch.
template <int FAM, int GS>
__device__ __forceinline__ void rmsnorm_quantize(const float *xv, float *xb, const float *w, float eps, int n,
                                                 int8_t *xq, float *xs) {
    __shared__ float s_inv;
    __syncthreads();
    for (int j = threadIdx.x; j < n; j += blockDim.x) xb[j] = __fmul_rn(xv[j], xv[j]);
    __syncthreads();
    if (threadIdx.x == 0) {
        float ss = chain_sum(xb, n);
        ss = __fdiv_rn(ss, (float)n);
        ss = __fadd_rn(ss, eps);
        s_inv = __frcp_rn(__fsqrt_rn(ss));  // 1.0f / sqrtf(...): same value
    }
    __syncthreads();
    const float s = s_inv;
    for (int j = threadIdx.x; j < n; j += blockDim.x) xb[j] = __fmul_rn(w[j], __fmul_rn(s, xv[j]));
    __syncthreads();
    quantize_to_global<FAM, GS>(xb, n, xq, xs);
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
// embedding row of the current token (qwen.c:498-501 with fp16 scales per 32, runq.c:490-492 with fp32 scales per
// group of gs), exact in fp32; also clears the head's argmax key.
template <int FAM>
__global__ void embed_kernel(const int8_t *emb_q, const void *emb_s, float *x, int dim, int gs, State *st,
                             unsigned long long *stamp) {
    allow_consumer();
    wait_for_producer();
    stamp_start(stamp);
    const int tok = __ldcg(&st->token);
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i == 0) st->key = 0ull;
    if (i < dim) {
        const size_t r = (size_t)tok * dim, g = (r + i) / gs;
        const float s = FAM == kRunq ? static_cast<const float *>(emb_s)[g]
                                     : scale_from_f16(static_cast<const uint16_t *>(emb_s)[g]);
        x[i] = __fmul_rn(__int2float_rn(emb_q[r + i]), s);
    }
    stamp_end(stamp);
}

// ---------------------------------------------------------------------------------------------------------------
enum Epilogue : int {
    kEpiStore = 0,     // out[row] = v
    kEpiResidual = 1,  // out[row] += v                                              (qwen.c:551, :565)
    kEpiSwiGLU = 2,    // tile = rows of w1 then the same rows of w3; out[row] = silu(g) * u   (qwen.c:558-562,
                       //                                                                      runq.c:588-596)
};

enum Prologue : int {
    kProQuantized = 0,  // xq/xs given (int8 + scales)
    kProQuant = 1,      // quantize the fp32 vector src                            (qwen.c:549, :563)
    kProNorm = 2,       // rmsnorm src with norm_w, then quantize                  (qwen.c:516-517, :554-555)
};

enum Tail : int {
    kTailNone = 0,
    kTailNormQuant = 1,  // rmsnorm(out) + quantize into tail_xq/xs               (qwen.c:569-570)
};

struct DecodeParams {
    const uint8_t *w[3];
    const void *ws[3];  // fp16 (kQwen) or fp32 (kRunq) scales
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
    const int32_t *head_ids;  // null: the argmax row is the token
    int *ids;
    int cap;
    unsigned long long *stamp;  // this kernel's two timing slots (stamp_start / stamp_end), or null
    // bytes that a later kernel will stream (the head's weights), prefetched into L2 by this kernel's CTAs before
    // they wait for the previous kernel, or null: the decode step leaves HBM mostly idle, so the head can be read
    // from L2 instead of waiting on HBM when its turn comes
    const uint8_t *l2_pf;
    size_t l2_pf_bytes;
};

// Asks L2 to fetch [p, p + bytes) (p 16-byte aligned, bytes a multiple of 16): a hint, no data comes back.
__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// This CTA's share of an L2 prefetch of [base, base + bytes): one thread issues it in 64 KB pieces.
__device__ __forceinline__ void prefetch_share_l2(const uint8_t *base, size_t bytes) {
    if (!base || threadIdx.x != 0) return;
    const size_t per = ((bytes + gridDim.x - 1) / gridDim.x + 15) & ~(size_t)15;
    const size_t b0 = per * blockIdx.x, b1 = min(b0 + per, bytes & ~(size_t)15);
    for (size_t o = b0; o < b1; o += 65536) prefetch_l2(base + o, (uint32_t)min((size_t)65536, b1 - o));
}

// Bytes of a decode matvec CTA's per-group activation scales and int4 offset sums, padded to 16 so that the
// product rows after them are 16-byte aligned.
__host__ __device__ constexpr size_t scale_bytes(int ng) { return ((size_t)ng * 8 + 15) & ~(size_t)15; }

// Activation planes of a decode matvec CTA: even/odd element planes for int4 weights, one plane per 16-byte chunk
// of a group for int8 weights (n bytes either way).
template <int BITS, int GS>
__host__ __device__ constexpr int activation_planes() { return BITS == 4 ? 2 : GS / 16; }

template <int BITS, int FAM, int GS, int EPI, int PRO, int TAIL, int UPT>
__global__ void __launch_bounds__(kThreads) decode_matvec_kernel(const DecodeParams p) {
    static_assert(FAM == kQwen || BITS == 8, "runq weights are int8");
    static_assert(GS == 32 || (GS == 64 && BITS == 8), "groups of 32, or 64 for int8 weights");
    constexpr int GB = GS * BITS / 8;  // weight bytes per group
    constexpr int WC = GB / 16;
    constexpr int XP = activation_planes<BITS, GS>();
    extern __shared__ __align__(16) uint8_t smem[];
    const int n = p.n, ng = n / GS, tid = threadIdx.x;
    const int row0 = blockIdx.x * p.rt;
    const int rows = min(p.rt, p.d - row0);
    const int vrows = EPI == kEpiSwiGLU ? 2 * rows : rows;
    const int units = vrows * ng;

    // 1. this tile's weights and scales into registers: they do not depend on any earlier kernel. Each unit's
    //    group and product slot are found here too, so that the product loop after the wait does no division.
    const int ps = prod_stride(ng);
    uint4 wv[UPT][WC];
    uint32_t hs[UPT];  // the scale's bits: fp16 (kQwen) or fp32 (kRunq), converted where it is used
    int ug[UPT], uslot[UPT];  // group of the unit, and its product's index vr * ps + g
#pragma unroll
    for (int k = 0; k < UPT; k++) {
        const int u = tid + k * kThreads;
        ug[k] = 0;
        uslot[k] = 0;
        if (u < units) {
            const int vr = u / ng, g = u - vr * ng;
            ug[k] = g;
            uslot[k] = vr * ps + g;
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
            const void *sb = m == 0 ? p.ws[0] : (m == 1 ? p.ws[1] : p.ws[2]);
            const size_t idx = (size_t)r * ng + g;
#pragma unroll
            for (int c = 0; c < WC; c++) wv[k][c] = ld_weights(wb + idx * GB + 16 * c);
            hs[k] = FAM == kRunq ? __float_as_uint(ld_f32(static_cast<const float *>(sb) + idx))
                                 : ld_u16(static_cast<const uint16_t *>(sb) + idx);
        }
    }
    prefetch_share_l2(p.l2_pf, p.l2_pf_bytes);
    // the rmsnorm weights this thread applies (constants), also before the wait
    float4 nw4[kNormPasses];
    if (PRO == kProNorm) norm_weights_for_planes<GS>(p.norm_w, n, nw4);
    if (EPI == kEpiStore) allow_consumer();
    wait_for_producer();
    stamp_start(p.stamp);
    // the residual's current value, loaded now so its latency overlaps the prologue
    float old = 0.0f;
    if (EPI == kEpiResidual && tid < rows) old = __ldcg(p.out + row0 + tid);

    // 2. this kernel's int8 input in shared-memory planes: from the previous kernel's int8 output, or quantized
    //    (after an rmsnorm) from its fp32 output by this CTA
    uint4 *xplane = reinterpret_cast<uint4 *>(smem);
    float *xs_s = reinterpret_cast<float *>(xplane + XP * ng);
    int *xsum_s = reinterpret_cast<int *>(xs_s + ng);
    // the products start on 16 bytes, as the fold reads them 16 bytes at a time: xs and xsum take 8 * ng bytes,
    // padded by 8 when ng is odd
    float *prod = reinterpret_cast<float *>(xsum_s + ng + 2 * (ng & 1));
    if (PRO == kProQuantized) {
        for (int c = tid; c < n / 16; c += kThreads) {
            const uint4 a = __ldcg(reinterpret_cast<const uint4 *>(p.xq) + c);
            const int g = c / (GS / 16), k = c % (GS / 16);
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
        for (int g = tid; g < ng; g += kThreads) xs_s[g] = __ldcg(p.xs + g);
    } else {
        // the fp32 input (and, for an rmsnorm, its squares then the normalized values) after the product stage,
        // addressed from the shared array itself so that every access compiles to a shared-memory load (a
        // pointer that went through an integer cast would be generic, and the in-order sum would run at the
        // generic load's latency)
        const size_t stage =
            (size_t)XP * ng * 16 + scale_bytes(ng) + (size_t)(EPI == kEpiSwiGLU ? 2 * p.rt : p.rt) * ps * 4;
        float *xv = reinterpret_cast<float *>(smem + ((stage + 15) & ~(size_t)15));
        const float4 z = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (PRO == kProNorm) {  // qwen.c:337-344, runq.c:394-407
            float *xn = xv + n;  // the squares, written in the same pass that stages x
            __shared__ float s_inv;
            for (int j = tid; j < n / 4; j += kThreads) {
                const float4 f = ld_cg4(p.src + 4 * j);
                reinterpret_cast<float4 *>(xv)[j] = f;
                reinterpret_cast<float4 *>(xn)[j] =
                    make_float4(__fmul_rn(f.x, f.x), __fmul_rn(f.y, f.y), __fmul_rn(f.z, f.z), __fmul_rn(f.w, f.w));
            }
            __syncthreads();
            if (tid == 0) {
                float ss = chain_sum(xn, n);
                ss = __fdiv_rn(ss, (float)n);
                ss = __fadd_rn(ss, p.eps);
                s_inv = __frcp_rn(__fsqrt_rn(ss));  // 1.0f / sqrtf(...): same value
            }
            __syncthreads();
            // normalized element by element inside the quantize (qwen.c:343's o[j] = w[j] * (ss * x[j]))
            quantize_to_planes<BITS, FAM, GS, true>(xv, n, reinterpret_cast<uint8_t *>(xplane), xs_s, xsum_s, nw4[0],
                                                    nw4[1], s_inv);
        } else if (ng <= kThreads / (GS / 4)) {
            // one pass of the quantize covers every group: each thread reads its own elements from L2, no staging
            quantize_to_planes<BITS, FAM, GS, false, true>(p.src, n, reinterpret_cast<uint8_t *>(xplane), xs_s, xsum_s,
                                                           z, z, 0.0f);
        } else {
            for (int j = tid; j < n / 4; j += kThreads) reinterpret_cast<float4 *>(xv)[j] = ld_cg4(p.src + 4 * j);
            __syncthreads();
            if (GS == 32 && ng > kThreads / 8)
                quantize_to_planes_wide<BITS, FAM>(xv, n, reinterpret_cast<uint8_t *>(xplane), xs_s, xsum_s);
            else
                quantize_to_planes<BITS, FAM, GS, false>(xv, n, reinterpret_cast<uint8_t *>(xplane), xs_s, xsum_s, z,
                                                         z, 0.0f);
        }
    }
    __syncthreads();
    if (BITS == 4 && PRO == kProQuantized) {  // the group sums (the quantizing prologues wrote them already)
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
        if (tid + k * kThreads < units) {
            const int g = ug[k];
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
                for (int c = 0; c < WC; c++) {
                    const uint4 a = xplane[c * ng + g];
                    acc = __dp4a((int)wv[k][c].x, (int)a.x, acc);
                    acc = __dp4a((int)wv[k][c].y, (int)a.y, acc);
                    acc = __dp4a((int)wv[k][c].z, (int)a.z, acc);
                    acc = __dp4a((int)wv[k][c].w, (int)a.w, acc);
                }
            }
            const float wscale = FAM == kRunq ? __uint_as_float(hs[k]) : scale_from_f16(hs[k]);
            prod[uslot[k]] = __fmul_rn(__fmul_rn(__int2float_rn(acc), wscale), xs_s[g]);
        }
    }
    __syncthreads();

    // Let the next kernel launch now (its CTAs prefetch their weights and then wait for this one). Launched
    // earlier, their resident CTAs slow this kernel's serial prologue (measured: 1,240 tok/s with the trigger at
    // the top, 1,421 here). The qkv kernel (the only one that stores its output plainly) is the exception: its
    // consumer is the 14-CTA attention, whose pre-wait loads of the cache are worth starting early.
    if (EPI != kEpiStore) allow_consumer();

    // 4. in-order fold of each virtual row, epilogue
    float v = 0.0f;
    if (tid < vrows) v = chain_sum_padded(prod + tid * ps, ng);  // rows are padded to a multiple of 4
    if (EPI == kEpiStore) {
        if (tid < rows) p.out[row0 + tid] = v;
    } else if (EPI == kEpiResidual) {
        if (tid < rows) p.out[row0 + tid] = __fadd_rn(old, v);
    } else if (EPI == kEpiSwiGLU) {
        // the tile's at most 16 gate rows and their up rows were folded by warp 0: lane r takes row r's up value
        // from lane rows + r
        if (tid < 32) {
            const float u = __shfl_sync(0xffffffffu, v, (tid + rows) & 31);
            if (tid < rows) {
                const float gv = __fmul_rn(v, __frcp_rn(__fadd_rn(1.0f, expf_ref(-v, p.et))));  // 1.0f / (...)
                p.out[row0 + tid] = __fmul_rn(gv, u);
            }
        }
    }

    // 5. the last CTA prepares the next kernel's input
    if (TAIL == kTailNone || !last_cta(p.counter)) {
        stamp_end(p.stamp);
        return;
    }
    float *sm = reinterpret_cast<float *>(smem);
    if (TAIL == kTailNormQuant) {
        for (int j = tid; j < p.d / 4; j += kThreads) reinterpret_cast<float4 *>(sm)[j] = ld_cg4(p.out + 4 * j);
        rmsnorm_quantize<FAM, GS>(sm, sm + p.d, p.tail_norm, p.eps, p.d, p.tail_xq, p.tail_xs);
    }
    stamp_end(p.stamp);
}

// The head's argmax key of logit v of row `row`: (v as an order-preserving integer << 32) | ~row, so that the
// largest key is the largest logit and, among equal logits, the first row, as the reference's scan with a strict
// `>` keeps (qwen.c:591-598, runq.c:843-854). -0 ties with +0, as `>` sees them. A NaN logit never wins, except
// at row 0: the scan starts from logit 0 and no comparison with a NaN succeeds, so a NaN there is the answer
// whatever follows; its all-ones key beats every ordered value and names row 0.
__device__ __forceinline__ unsigned long long head_key(float v, int row) {
    const float c = v == 0.0f ? 0.0f : v;
    const uint32_t b = __float_as_uint(c);
    const uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    if (c == c) return ((unsigned long long)ord << 32) | (uint32_t)(~(uint32_t)row);
    return row == 0 ? ~0ull : 0ull;
}

// The head (qwen.c's trimmed Q8 head, qwen.c:571; runq.c's classifier, runq.c:611): logits of every row, their
// argmax, and the next token (qwen.c:677-683: the prompt's next token, else head_ids[argmax]; runq.c:1006-1012: the
// argmax row itself). Persistent like matvec_kernel: one CTA per resident slot, each owning a balanced block of
// rows streamed in tiles of p.rt rows with the int8 input staged once; each thread keeps the best key of the rows it
// folded, one atomicMax per warp publishes them, and the last CTA to finish picks the token. The head's weights
// were prefetched into L2 during the last layer (DecodeParams::l2_pf of an earlier kernel), so the tiles stream
// from L2.
template <int FAM, int GS>
__global__ void __launch_bounds__(kThreads, 4) head_kernel(const DecodeParams p) {
    constexpr int FMT = FAM == kRunq ? kQ8F32 : kQ8F16;
    constexpr int XC = GS / 16;
    extern __shared__ __align__(16) uint8_t smem[];
    const int n = p.n, ng = n / GS, tid = threadIdx.x;
    const MatvecSmem<GS> sm(smem, ng);
    MatvecParams mp = {};
    mp.w = p.w[0];
    mp.ws = p.ws[0];
    mp.n = n;
    mp.d = p.d;
    mp.rt = p.rt;
    int r0, r1;
    cta_rows(p.d, blockIdx.x, gridDim.x, r0, r1);
    wait_for_producer();
    stamp_start(p.stamp);
    // the int8 input (written by the previous kernel: L2 loads) into the chunk planes, and its scales
    for (int c = tid; c < n / 16; c += kThreads) {
        const int g = c / XC, k = c % XC;
        sm.xplane[k * ng + g] = __ldcg(reinterpret_cast<const uint4 *>(p.xq) + c);
    }
    for (int g = tid; g < ng; g += kThreads) sm.xs[g] = __ldcg(p.xs + g);
    __syncthreads();
    unsigned long long key = 0ull;
    for (int row0 = r0; row0 < r1; row0 += p.rt) {
        stream_tile<FMT, GS>(mp, sm, row0, min(p.rt, r1 - row0), [&](int row, float v) {
            p.out[row] = v;
            const unsigned long long k = head_key(v, row);
            key = k > key ? k : key;
        });
        __syncthreads();  // the next tile rewrites the product buffer
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) {
        const unsigned long long o = __shfl_xor_sync(0xffffffffu, key, off);
        key = o > key ? o : key;
    }
    if ((tid & 31) == 0 && key) atomicMax(&p.st->key, key);
    if (!last_cta(p.counter)) {
        stamp_end(p.stamp);
        return;
    }
    if (tid == 0) {
        State *st = p.st;
        const int pos = st->pos;
        const unsigned long long best = atomicAdd(&st->key, 0ull);
        // no key cannot happen (a NaN logit 0 gives the all-ones key); kept as row 0, the reference's answer
        const int row = best ? (int)(~(uint32_t)(best & 0xffffffffu)) : 0;
        st->last_row = row;
        if (st->n_prompt >= 0) {
            int next;
            if (pos + 1 < st->n_prompt) {
                next = p.prompt[pos + 1];
            } else {
                next = p.head_ids ? p.head_ids[row] : row;
                if (st->n_gen < p.cap) p.ids[st->n_gen] = next;
                st->n_gen++;
            }
            st->token = next;
        }
        st->pos = pos + 1;
    }
    stamp_end(p.stamp);
}

// Dynamic shared memory of decode_matvec_kernel for groups of gs: the product stage (plus x and the normalized x
// for an rmsnorm prologue), or the tail's staging if larger. The activation planes take n bytes for every format.
inline size_t decode_smem_bytes(int n, int gs, int rt, int epi, int pro, int tail, int d) {
    const int ng = n / gs;
    const int vmax = epi == kEpiSwiGLU ? 2 * rt : rt;
    size_t b = (size_t)n + scale_bytes(ng) + (size_t)vmax * prod_stride(ng) * 4;
    if (pro != kProQuantized) b = ((b + 15) & ~(size_t)15) + (size_t)(pro == kProNorm ? 2 : 1) * n * 4;
    size_t t = tail == kTailNormQuant ? (size_t)2 * d * 4 : 0;
    return b > t ? b : t;
}

// ---------------------------------------------------------------------------------------------------------------
// attention for one query head (qwen.c:521-546; runq.c:506-567): the biases and NeoX RoPE (pairs i, i + hs/2) of
// qwen.c, or runq.c's interleaved RoPE (pairs 2i, 2i + 1) without biases; the KV-cache write of this position,
// scores q.k / sqrt(hs) in order over the head's elements, softmax in order, weighted values in order of position.
// The cached values of this head's kv head are staged in shared memory (cp.async, double buffered in chunks of
// kVChunk positions) while the scores are computed.
constexpr int kVChunk = 256;

struct AttnParams {
    const float *qkv;   // raw outputs of the qkv matvec: q (dim) | k (kv_dim) | v (kv_dim)
    const float *bq, *bk, *bv;  // kQwen only
    const float *rope;  // per position: cos[hs/2] then sin[hs/2] of each rotated pair
    float *kcache, *vcache;  // this layer's (ctx, kv_dim)
    float *xb;          // dim outputs
    int dim, kv_dim, kv_mul, ctx;
    State *st;
    ExpTable et;
    unsigned long long *stamp;  // timing slots (stamp_start / stamp_end), or null
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

// acc + a_0 v_0 + a_1 v_1 + ... + a_{nt-1} v_{nt-1}, added in order (v_t = vb[t * HS]). The products are off the
// dependent chain of adds and are formed in blocks of 8 two blocks ahead, so the chain runs at the latency of one
// fp32 add per position (the same scheme as chain_sum).
template <int HS>
__device__ __forceinline__ float weighted_chain(float acc, const float *a, const float *vb, int nt) {
    int t = 0;
    const int n8 = nt & ~7;
    // the last nt - n8 (< 8) products are formed first, off the chain (indices clamped into [0, nt))
    float tail[7];
#pragma unroll
    for (int i = 0; i < 7; i++) {
        const int j = n8 + i < nt ? n8 + i : 0;
        tail[i] = __fmul_rn(a[j], vb[j * HS]);
    }
    if (n8 == 8) {
        float p0[8];
#pragma unroll
        for (int i = 0; i < 8; i++) p0[i] = __fmul_rn(a[i], vb[i * HS]);
#pragma unroll
        for (int i = 0; i < 8; i++) acc = __fadd_rn(acc, p0[i]);
        t = 8;
    } else if (n8 >= 16) {
        float p0[8], p1[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            p0[i] = __fmul_rn(a[i], vb[i * HS]);
            p1[i] = __fmul_rn(a[8 + i], vb[(8 + i) * HS]);
        }
        for (; t < n8; t += 8) {
            const int tn = t + 16 < n8 ? t + 16 : t;  // stays inside [0, n8)
            float p2[8];
#pragma unroll
            for (int i = 0; i < 8; i++) p2[i] = __fmul_rn(a[tn + i], vb[(tn + i) * HS]);
#pragma unroll
            for (int i = 0; i < 8; i++) acc = __fadd_rn(acc, p0[i]);
#pragma unroll
            for (int i = 0; i < 8; i++) {
                p0[i] = p1[i];
                p1[i] = p2[i];
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 7; i++)
        if (n8 + i < nt) acc = __fadd_rn(acc, tail[i]);
    return acc;
}

template <int HS, int FAM>
__global__ void __launch_bounds__(kThreads) attention_kernel(const AttnParams p) {
    extern __shared__ __align__(16) float asm_[];
    float *q = asm_, *kc = q + HS, *vc = kc + HS;
    float *att = vc + HS;                                  // ctx scores
    float *vbuf = att + ((p.ctx + 3) & ~3);                // 2 x kVChunk x HS staged values
    __shared__ float red[kThreads / 32];
    __shared__ float s_sum;
    const int h = blockIdx.x, kvh = h / p.kv_mul, half = HS / 2, tid = threadIdx.x;
    // Everything up to the wait reads only what earlier steps wrote (the position, set by the previous step's
    // head kernel; the cache rows of earlier positions) or constants (RoPE table, biases). Within one step no
    // kernel writes them before this kernel has finished, so they are read before the qkv kernel completes.
    const int pos = __ldcg(&p.st->pos);
    const int nchunks = (pos + kVChunk - 1) / kVChunk;  // cached positions 0 .. pos-1
    if (nchunks > 0) stage_values<HS>(vbuf, p.vcache, p.kv_dim, kvh, 0, min(kVChunk, pos));
    cp_async_commit();
    // this thread's first cached key row
    float4 k4[HS / 4];
    if (tid < pos) {
        const float *kt = p.kcache + (size_t)tid * p.kv_dim + kvh * HS;
#pragma unroll
        for (int i = 0; i < HS / 4; i++) k4[i] = ld_cg4(kt + 4 * i);
    }
    const float *cs = p.rope + (size_t)pos * HS;
    // this thread's rotated pair (i0, i1): NeoX halves for qwen.c, neighbours for runq.c
    const int i0 = FAM == kRunq ? 2 * tid : tid, i1 = FAM == kRunq ? 2 * tid + 1 : tid + half;
    float rc = 0.0f, rs = 0.0f, bq0 = 0.0f, bq1 = 0.0f, bk0 = 0.0f, bk1 = 0.0f, bv0 = 0.0f;
    if (tid < half) {
        rc = cs[tid];
        rs = cs[half + tid];
        if (FAM == kQwen) {
            bq0 = p.bq[h * HS + i0];
            bq1 = p.bq[h * HS + i1];
            bk0 = p.bk[kvh * HS + i0];
            bk1 = p.bk[kvh * HS + i1];
        }
    }
    if (FAM == kQwen && tid < HS) bv0 = p.bv[kvh * HS + tid];
    wait_for_producer();
    stamp_start(p.stamp);
    const float *qr = p.qkv + h * HS, *kr = p.qkv + p.dim + kvh * HS, *vr = p.qkv + p.dim + p.kv_dim + kvh * HS;
    // qwen.c adds the biases to the raw outputs (qwen.c:521-524); runq.c rotates them as they are (runq.c:506-521)
    auto in = [](const float *r, int i, float bias) {
        return FAM == kQwen ? __fadd_rn(__ldcg(r + i), bias) : __ldcg(r + i);
    };
    if (tid < half) {
        float a = in(qr, i0, bq0), b = in(qr, i1, bq1);
        q[i0] = __fsub_rn(__fmul_rn(a, rc), __fmul_rn(b, rs));
        q[i1] = __fadd_rn(__fmul_rn(b, rc), __fmul_rn(a, rs));
        a = in(kr, i0, bk0);
        b = in(kr, i1, bk1);
        kc[i0] = __fsub_rn(__fmul_rn(a, rc), __fmul_rn(b, rs));
        kc[i1] = __fadd_rn(__fmul_rn(b, rc), __fmul_rn(a, rs));
    }
    if (tid < HS) vc[tid] = in(vr, tid, bv0);
    __syncthreads();
    if (h % p.kv_mul == 0 && tid < HS) {  // one writer per kv head
        p.kcache[(size_t)pos * p.kv_dim + kvh * HS + tid] = kc[tid];
        p.vcache[(size_t)pos * p.kv_dim + kvh * HS + tid] = vc[tid];
    }
    // scores: one position per thread, the head's HS products added in order; each thread keeps the largest of
    // its scores for the softmax
    const float scale = __fsqrt_rn((float)HS);
    float m = -INFINITY;
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
        const float a = __fdiv_rn(score, scale);
        att[t] = a;
        m = fmaxf(m, a);
    }
    // softmax (qwen.c:346-352, runq.c:409-427): max (order-free: the same value as the reference's scan), exp(x -
    // max), in-order sum, divide. Every thread combines the warps' maxima itself, and exponentiates only the
    // scores it wrote, so one barrier serves the max.
#pragma unroll
    for (int off = 16; off; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if ((tid & 31) == 0) red[tid >> 5] = m;
    __syncthreads();
    float mx = red[0];
#pragma unroll
    for (int w = 1; w < kThreads / 32; w++) mx = fmaxf(mx, red[w]);
    for (int t = tid; t <= pos; t += kThreads) att[t] = expf_ref(__fsub_rn(att[t], mx), p.et);
    __syncthreads();
    if (tid == 0) s_sum = chain_sum_padded(att, pos + 1);  // att holds a multiple of 4 floats
    __syncthreads();
    const float sum = s_sum;
    for (int t = tid; t <= pos; t += kThreads) att[t] = __fdiv_rn(att[t], sum);
    // The next kernel may launch: here for runq models; for Qwen after the weighted values below, whose serial
    // chains the next kernel's early-resident CTAs slow down (measured: Qwen step 0.620 -> 0.607 ms when released
    // after them; stories15M 0.115 -> 0.116 ms, so it keeps the earlier release).
    if (FAM == kRunq) allow_consumer();
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
            const int t0 = c * kVChunk;
            acc = weighted_chain<HS>(acc, att + t0, vbuf + (c & 1) * kVChunk * HS + tid, min(kVChunk, pos - t0));
        }
        __syncthreads();
    }
    if (FAM == kQwen) allow_consumer();
    if (tid < HS) {
        acc = __fadd_rn(acc, __fmul_rn(att[pos], vc[tid]));
        p.xb[h * HS + tid] = acc;
    }
    stamp_end(p.stamp);
}

template <int HS>
inline size_t attention_smem_bytes(int ctx) {
    return (size_t)3 * HS * 4 + (size_t)((ctx + 3) & ~3) * 4 + (size_t)2 * kVChunk * HS * 4;
}

}  // namespace decode
}  // namespace mvb
