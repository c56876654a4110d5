// Device-resident Qwen2 decode over the group-quantized matvec (the reference's token loop, qwen/qwen.c:490-573
// and :669-712, moved onto the B200 so the matvecs run back to back instead of one host round trip each).
//
// One forward step is a fixed sequence of 122 kernels (for 24 layers), captured once into a CUDA graph:
//   embed                       x = dequantized embedding row of the current token          qwen.c:498-501
//   per layer:
//     qkv  (fused matvec)       rmsnorm(x) -> quantize -> [wq; wk; wv] rows, raw outputs     qwen.c:516-520
//     attention (per q head)    + biases, NeoX RoPE, KV-cache write, softmax attention       qwen.c:521-546
//     o    (fused matvec)       quantize(xb) -> wo, x += out                                 qwen.c:549-551
//     gate/up (fused matvec)    rmsnorm(x) -> quantize -> w1, w3 rows paired, SwiGLU -> hb    qwen.c:554-562
//     down (fused matvec)       quantize(hb) -> w2, x += out; after the last layer its last  qwen.c:563-565,
//                               CTA also does the final rmsnorm + quantize                   :569-570
//   head (persistent matvec)    Q8 head rows -> logits, argmax -> atomicMax; its last CTA   qwen.c:571, 591-598,
//                               picks the next token (prompt[pos+1], else head_ids[argmax])  :677-683
//                               (the last layer's qkv kernel prefetched the head into L2)
// The step reads the token and the position from device memory, so the same graph serves every position and
// a whole generation is the graph launched once per position with no host work in between. The prompt is fed
// in batches instead (prefill_batch: tensor-core matmuls, prefill_kernels.cuh), which writes the same KV cache.
//
// Arithmetic follows qwen.c operation by operation: no fused multiply-adds (the library is built with
// -fmad=false and uses explicitly rounded intrinsics), sums in the reference's order (rmsnorm's sum of squares,
// attention dots, the softmax denominator and the weighted value sum are all sequential loops there and here),
// RoPE angles from the host's double-precision pow/cos/sin exactly as qwen.c:504-508 computes them, and expf
// (softmax, SiLU) with the host C library's exact results (expf_ref.h), so the step reproduces qwen.c's logits
// bit for bit.
//
// The same runtime decodes runq.c's int8 models (mvb_runq_load): the kernel sequence is the same, with runq.c's
// arithmetic where it differs (runq.c:477-614): int8 weights with fp32 scales in groups of 32 or 64, activation
// quantization by division, rmsnorm eps 1e-5, interleaved RoPE from the host C library's float powf/cosf/sinf
// (runq.c:506-521), no biases, and a classifier whose argmax row is the token (runq.c:843-854). A .qwb model can
// also use its tied embedding as a full-vocabulary head (mvb_qwen_full_head).
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <time.h>
#include <unistd.h>

#include <map>
#include <mutex>
#include <vector>

#include "../../include/matvec_b200.h"
#include "decode_kernels.cuh"
#include "expf_ref.h"
#include "prefill_kernels.cuh"
#include "matvec_kernels.cuh"
#include "mvb_runtime.h"

namespace mvb {
namespace decode {

constexpr int kMaxDim = 2048;     // largest dim the norm kernels stage in shared memory
constexpr int kMaxCtx = 8192;     // largest context (attention scores live in shared memory)

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
        inv_rms = __frcp_rn(__fsqrt_rn(ss));  // 1.0f / sqrtf(...): the correctly rounded reciprocal
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
        uint32_t q4[8];
        xs[g] = quantize_group<32>(xb, g, kXQuantizeQwen, q4);
        uint4 *dst = reinterpret_cast<uint4 *>(xq + 32 * g);  // xq is 16-byte aligned
        dst[0] = make_uint4(q4[0], q4[1], q4[2], q4[3]);
        dst[1] = make_uint4(q4[4], q4[5], q4[6], q4[7]);
    }
    allow_consumer();
}

// ---------------------------------------------------------------------------------------------------------------
struct Config {
    int dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, head_k, max_seq_len, group_size, emb_bits;
    float rope_theta, rms_eps;
};

struct Mat {
    const uint8_t *w;
    const void *s;  // fp16 scales (kQwen) or fp32 scales (kRunq), one per group of 32
};

struct Model {
    Config c;
    int family = kQwen;  // kQwen: a .qwb model for qwen.c; kRunq: a runq v2 model for runq.c
    int hs = 0, kv_dim = 0, ctx = 0;
    int device = 0;
    bool pdl = true;
    cudaStream_t stream = nullptr;
    cudaGraphExec_t graph = nullptr;
    uint8_t *image = nullptr;  // the weights on the device: the whole .qwb at its own offsets, or the runq arena
    size_t image_bytes = 0;
    const float *attn_norm = nullptr, *ffn_norm = nullptr, *bq = nullptr, *bk = nullptr, *bv = nullptr,
                *out_norm = nullptr;
    const int32_t *head_ids = nullptr;  // kQwen: token id of each head row; kRunq: none (row = token)
    int head_rows = 0;                  // rows of the head in use: head_k, or vocab_size for a full head
    Mat head_trim = {};                 // the file's head and its ids, kept while a full head is in use
    const int32_t *ids_trim = nullptr;
    std::vector<Mat> wq, wk, wv, wo, w1, w2, w3;
    Mat head, emb;
    float *x = nullptr, *xb = nullptr, *qkv = nullptr, *hb = nullptr, *logits = nullptr, *kcache = nullptr,
          *vcache = nullptr, *rope = nullptr;
    // the final normalized x, quantized once for the head by the last layer's down projection
    int8_t *xq_n = nullptr;
    float *xs_n = nullptr;
    int *counters = nullptr;  // one last-CTA counter per kernel of the step
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
    // the step again as the graph runs it (programmatic overlap included), every kernel stamping %globaltimer
    // into its two slots of `stamps` (stamp_start / stamp_end): where the step's time goes, kernel by kernel
    cudaGraphExec_t stamp_graph = nullptr;
    unsigned long long *stamps = nullptr;
    bool stamping = false;  // set while the stamped copy is captured
    struct Info { const char *kind; int layer; };
    std::vector<Info> info;  // one per kernel of the step, in launch order
    // batched prefill buffers (allocated on first use): up to `cap` tokens per batch
    struct Batch {
        int cap = 0;
        float *x = nullptr, *qkv = nullptr, *qb = nullptr, *att = nullptr, *out = nullptr, *h1 = nullptr,
              *h3 = nullptr, *xs = nullptr;
        int8_t *xq = nullptr;
        // matmuls of one input run side by side (q, k, v; gate, up): two more streams, forked from and joined to
        // the model's stream by events
        cudaStream_t side[2] = {nullptr, nullptr};
        cudaEvent_t fork = nullptr, join[2] = {nullptr, nullptr};
    } pf;
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

// Rows per tile for a decode matvec: `target`, or fewer so that the tile's groups (of gs) fit UPT per thread.
static int decode_rt(int target, int n, int gs, int upt, bool pair) {
    const int per_row = (n / gs) * (pair ? 2 : 1);
    const int lim = kThreads * upt / per_row;
    return target < lim ? target : lim;
}

// The head: a persistent grid of one CTA per resident slot (at most one per row), tiles of p.rt rows.
template <int FAM, int GS>
static cudaError_t launch_head(Model &m, DecodeParams p, int *count) {
    const size_t smem = matvec_smem_bytes(p.n, GS, p.rt);
    const int slots = resident_slots((const void *)head_kernel<FAM, GS>, smem);
    p.counter = m.counters + *count;
    p.stamp = m.stamping ? m.stamps + 2 * *count : nullptr;
    (*count)++;
    return launch(head_kernel<FAM, GS>, dim3(p.d < slots ? p.d : slots), dim3(kThreads), smem, m.stream, m.pdl, p);
}

template <int BITS, int FAM, int GS, int EPI, int PRO, int TAIL, int UPT>
static cudaError_t launch_decode(Model &m, DecodeParams p, int *count) {
    const size_t smem = decode_smem_bytes(p.n, GS, p.rt, EPI, PRO, TAIL, p.d);
    if (EPI == kEpiSwiGLU && p.rt > 16) return cudaErrorInvalidValue;  // the epilogue folds in one warp
    p.counter = m.counters + *count;
    p.stamp = m.stamping ? m.stamps + 2 * *count : nullptr;
    (*count)++;
    return launch(decode_matvec_kernel<BITS, FAM, GS, EPI, PRO, TAIL, UPT>, dim3((p.d + p.rt - 1) / p.rt),
                  dim3(kThreads), smem, m.stream, m.pdl, p);
}

// Head sizes the attention kernel is built for, per family (the loaders refuse others).
template <int HS, int FAM>
static cudaError_t set_attention_smem() {
    // the attribute is per kernel, not per model: set it for the largest context any model may have, so that
    // loading a model with a smaller context never lowers it under another model's launches
    return cudaFuncSetAttribute(attention_kernel<HS, FAM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)attention_smem_bytes<HS>(kMaxCtx));
}

static cudaError_t set_attention_smem_all() {
    cudaError_t e;
    if ((e = set_attention_smem<64, kQwen>()) != cudaSuccess || (e = set_attention_smem<32, kRunq>()) != cudaSuccess ||
        (e = set_attention_smem<48, kRunq>()) != cudaSuccess || (e = set_attention_smem<64, kRunq>()) != cudaSuccess)
        return e;
    return cudaSuccess;
}

template <int FAM>
static cudaError_t launch_attention(Model &m, const AttnParams &a) {
    const dim3 grid(m.c.n_heads), block(kThreads);
    const cudaStream_t s = m.stream;
    switch (FAM == kQwen ? 64 : m.hs) {
        case 32: return launch(attention_kernel<32, FAM>, grid, block, attention_smem_bytes<32>(m.ctx), s, m.pdl, a);
        case 48: return launch(attention_kernel<48, FAM>, grid, block, attention_smem_bytes<48>(m.ctx), s, m.pdl, a);
        default: return launch(attention_kernel<64, FAM>, grid, block, attention_smem_bytes<64>(m.ctx), s, m.pdl, a);
    }
}

// Enqueues one forward step on m.stream (captured into a graph by the caller). With `ev`, records ev[k] before
// kernel k and ev[count] after the last one; `info` receives each kernel's kind and layer; with `trace`, the
// residual stream x is copied out after the embedding (slot 0) and after each layer's attention (2l + 1) and FFN
// (2l + 2). The kernel sequence is the same for both families (qwen.c:490-573, runq.c:477-614); they differ in
// the weight format (Q4 + fp16 scales vs Q8 + fp32 scales), the group size (32; runq also 64), the quantization
// rule, RoPE, biases and the head.
template <int FAM, int GS>
static cudaError_t enqueue_step_family(Model &m, int *count, cudaEvent_t *ev, std::vector<Model::Info> *info,
                                       float *trace) {
    constexpr int BITS = FAM == kQwen ? 4 : 8;  // layer matrices
    // groups per thread: a group of 64 carries twice the bytes of a group of 32, so half as many fit the registers
    constexpr int U1 = 1, U4 = GS == 64 ? 2 : 4, U5 = GS == 64 ? 3 : 5;
    const Config &c = m.c;
    cudaError_t e;
    *count = 0;
    // inside stream capture a plain event record is only a dependency marker; External makes it a graph node
    auto mark = [&](const char *kind, int layer) -> cudaError_t {
        if (info) info->push_back(Model::Info{kind, layer});
        return ev ? cudaEventRecordWithFlags(ev[*count], m.stream, cudaEventRecordExternal) : cudaSuccess;
    };
    auto snap = [&](int slot) -> cudaError_t {
        return trace ? cudaMemcpyAsync(trace + (size_t)slot * c.dim, m.x, c.dim * 4, cudaMemcpyDeviceToDevice,
                                       m.stream)
                     : cudaSuccess;
    };
    const int dim = c.dim, hid = c.hidden_dim, kv = m.kv_dim, L = c.n_layers;
    if ((e = mark("embed", -1)) != cudaSuccess) return e;
    e = launch(embed_kernel<FAM>, dim3((dim + kThreads - 1) / kThreads), dim3(kThreads), 0, m.stream, m.pdl,
               (const int8_t *)m.emb.w, m.emb.s, m.x, dim, GS, m.st,
               m.stamping ? m.stamps + 2 * *count : (unsigned long long *)nullptr);
    (*count)++;
    if (e != cudaSuccess || (e = snap(0)) != cudaSuccess) return e;
    for (int l = 0; l < L; l++) {
        // qkv: rmsnorm + quantize of x in every CTA, then [wq; wk; wv] rows
        DecodeParams p = {};
        p.w[0] = m.wq[l].w; p.ws[0] = m.wq[l].s; p.rows[0] = dim;
        p.w[1] = m.wk[l].w; p.ws[1] = m.wk[l].s; p.rows[1] = kv;
        p.w[2] = m.wv[l].w; p.ws[2] = m.wv[l].s; p.rows[2] = kv;
        p.n = dim; p.d = dim + 2 * kv; p.rt = decode_rt(8, dim, GS, U1, false);
        p.src = m.x; p.norm_w = m.attn_norm + (size_t)l * dim; p.eps = c.rms_eps; p.out = m.qkv; p.st = m.st;
        if (l == L - 1) {  // the head's weights and scales into L2 while the last layer runs
            const uint8_t *hw = m.head.w, *hs = static_cast<const uint8_t *>(m.head.s);
            const size_t wb = (size_t)m.head_rows * dim, sb = (size_t)m.head_rows * (dim / GS) * (FAM == kRunq ? 4 : 2);
            const uint8_t *lo = hw < hs ? hw : hs, *hi = hw + wb > hs + sb ? hw + wb : hs + sb;
            p.l2_pf = lo;
            p.l2_pf_bytes = (size_t)(hi - lo);
        }
        if ((e = mark("qkv", l)) != cudaSuccess ||
            (e = launch_decode<BITS, FAM, GS, kEpiStore, kProNorm, kTailNone, U1>(m, p, count)) != cudaSuccess)
            return e;
        // attention
        AttnParams a = {};
        a.qkv = m.qkv;
        if (FAM == kQwen) {
            a.bq = m.bq + (size_t)l * dim; a.bk = m.bk + (size_t)l * kv; a.bv = m.bv + (size_t)l * kv;
        }
        a.rope = m.rope;
        a.kcache = m.kcache + (size_t)l * m.ctx * kv; a.vcache = m.vcache + (size_t)l * m.ctx * kv;
        a.xb = m.xb; a.dim = dim; a.kv_dim = kv; a.kv_mul = c.n_heads / c.n_kv_heads; a.ctx = m.ctx; a.st = m.st;
        a.et = m.et;
        a.stamp = m.stamping ? m.stamps + 2 * *count : nullptr;
        if ((e = mark("attention", l)) != cudaSuccess || (e = launch_attention<FAM>(m, a)) != cudaSuccess) return e;
        (*count)++;
        // o: quantize the attention output in every CTA, x += wo * it
        p = DecodeParams{};
        p.w[0] = m.wo[l].w; p.ws[0] = m.wo[l].s; p.rows[0] = dim;
        p.n = dim; p.d = dim; p.rt = decode_rt(8, dim, GS, U1, false);
        p.src = m.xb; p.out = m.x; p.st = m.st;
        if ((e = mark("o_proj", l)) != cudaSuccess ||
            (e = launch_decode<BITS, FAM, GS, kEpiResidual, kProQuant, kTailNone, U1>(m, p, count)) != cudaSuccess ||
            (e = snap(2 * l + 1)) != cudaSuccess)
            return e;
        // gate/up: rmsnorm + quantize of x in every CTA, paired rows, SwiGLU -> hb
        p = DecodeParams{};
        p.w[0] = m.w1[l].w; p.ws[0] = m.w1[l].s; p.rows[0] = hid;
        p.w[1] = m.w3[l].w; p.ws[1] = m.w3[l].s; p.rows[1] = hid;
        p.n = dim; p.d = hid; p.rt = decode_rt(16, dim, GS, U4, true);
        p.src = m.x; p.norm_w = m.ffn_norm + (size_t)l * dim; p.eps = c.rms_eps; p.out = m.hb; p.st = m.st;
        p.et = m.et;
        if ((e = mark("gate_up", l)) != cudaSuccess ||
            (e = launch_decode<BITS, FAM, GS, kEpiSwiGLU, kProNorm, kTailNone, U4>(m, p, count)) != cudaSuccess)
            return e;
        // down: quantize hb in every CTA, x += w2 * it; after the last layer, the last CTA normalizes x for the head
        p = DecodeParams{};
        p.w[0] = m.w2[l].w; p.ws[0] = m.w2[l].s; p.rows[0] = dim;
        p.n = hid; p.d = dim; p.rt = decode_rt(8, hid, GS, U5, false);
        p.src = m.hb; p.out = m.x; p.st = m.st;
        p.tail_norm = m.out_norm; p.eps = c.rms_eps; p.tail_xq = m.xq_n; p.tail_xs = m.xs_n;
        if ((e = mark("down", l)) != cudaSuccess) return e;
        e = l + 1 < L ? launch_decode<BITS, FAM, GS, kEpiResidual, kProQuant, kTailNone, U5>(m, p, count)
                      : launch_decode<BITS, FAM, GS, kEpiResidual, kProQuant, kTailNormQuant, U5>(m, p, count);
        if (e != cudaSuccess || (e = snap(2 * l + 2)) != cudaSuccess) return e;
    }
    // head (qwen.c's trimmed Q8 head, or runq.c's classifier): logits + argmax; the last CTA picks the next token
    DecodeParams p = {};
    p.w[0] = m.head.w; p.ws[0] = m.head.s; p.rows[0] = m.head_rows;
    p.n = dim; p.d = m.head_rows; p.rt = 32;
    p.xq = m.xq_n; p.xs = m.xs_n; p.out = m.logits; p.st = m.st;
    p.prompt = m.prompt; p.head_ids = m.head_ids; p.ids = m.ids; p.cap = m.ctx;
    if ((e = mark("head", -1)) != cudaSuccess || (e = launch_head<FAM, GS>(m, p, count)) != cudaSuccess) return e;
    if (ev) e = cudaEventRecordWithFlags(ev[*count], m.stream, cudaEventRecordExternal);
    return e;
}

static cudaError_t enqueue_step(Model &m, int *count, cudaEvent_t *ev = nullptr,
                                std::vector<Model::Info> *info = nullptr, float *trace = nullptr) {
    if (m.family == kQwen) return enqueue_step_family<kQwen, 32>(m, count, ev, info, trace);
    return m.c.group_size == 64 ? enqueue_step_family<kRunq, 64>(m, count, ev, info, trace)
                                : enqueue_step_family<kRunq, 32>(m, count, ev, info, trace);
}

// Algorithmic bytes of kernel k of the step at position `pos`: every byte the kernel must move at least once
// (weights and scales, activations in and out, norm weights, KV-cache rows read and written).
static double kernel_bytes(const Model &m, int k, int pos) {
    const Config &c = m.c;
    const double gs = c.group_size, dim = c.dim, hid = c.hidden_dim, kv = m.kv_dim, ng = dim / gs;
    const char *kind = m.info[k].kind;
    const bool runq = m.family == kRunq;
    const double sb = runq ? 4 : 2;  // bytes per weight scale
    // one layer matrix: Q4 + fp16 scales (qwen.c) or Q8 + fp32 scales (runq.c)
    auto mat = [&](double d, double n) { return d * n * (runq ? 1.0 : 0.5) + d * (n / gs) * sb; };
    if (!strcmp(kind, "embed")) return dim + ng * sb + dim * 4;
    // matvecs: weights + scales, int8 input + scales, outputs (read + write for residual updates); tails: the
    // vector they normalize or quantize, the norm weight, the int8 output
    const bool last = m.info[k].layer == c.n_layers - 1;
    if (!strcmp(kind, "qkv")) return mat(dim + 2 * kv, dim) + dim * 4 * 2 + (dim + 2 * kv) * 4;
    if (!strcmp(kind, "attention"))  // q/k/v in (+ biases), RoPE row, cached rows read, this row written, output
        return (dim + 2 * kv) * 4 * (runq ? 1 : 2) + m.hs * 4 + 2.0 * pos * kv * 4 + 2 * kv * 4 + dim * 4;
    if (!strcmp(kind, "o_proj")) return mat(dim, dim) + dim * 4 + dim * 8;
    if (!strcmp(kind, "gate_up")) return 2 * mat(hid, dim) + dim * 4 * 2 + hid * 4;
    if (!strcmp(kind, "down")) return mat(dim, hid) + hid * 4 + dim * 8 + (last ? dim * 4 * 2 + dim + ng * 4 : 0);
    if (!strcmp(kind, "head"))
        return (double)m.head_rows * dim + (double)m.head_rows * ng * sb + dim + ng * 4 + m.head_rows * 4.0;
    return 16;
}

static void destroy(Model *m) {
    if (!m) return;
    if (m->stream) cudaStreamSynchronize(m->stream);
    if (m->graph) cudaGraphExecDestroy(m->graph);
    if (m->prof_graph) cudaGraphExecDestroy(m->prof_graph);
    if (m->stamp_graph) cudaGraphExecDestroy(m->stamp_graph);
    for (cudaEvent_t e : m->prof_ev) cudaEventDestroy(e);
    if (m->ring) cudaFreeHost(m->ring);
    void *bufs[] = {m->image, m->x, m->xb, m->qkv, m->hb, m->logits, m->kcache, m->vcache, m->rope, m->xq_n,
                    m->xs_n, m->counters, m->prompt, m->ids, m->st, m->stamps, m->pf.x, m->pf.qkv, m->pf.qb, m->pf.att,
                    m->pf.out, m->pf.h1, m->pf.h3, m->pf.xs, m->pf.xq};
    for (void *b : bufs)
        if (b) cudaFree(b);
    for (int i = 0; i < 2; i++) {
        if (m->pf.side[i]) cudaStreamDestroy(m->pf.side[i]);
        if (m->pf.join[i]) cudaEventDestroy(m->pf.join[i]);
    }
    if (m->pf.fork) cudaEventDestroy(m->pf.fork);
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

constexpr int kBatchCap = 256;  // prompt tokens per batched prefill pass
constexpr int kGqaSmemMax = 200 * 1024;  // shared memory of the grouped prefill attention, at most

// Runs prompt tokens tokens[0 .. count-1] (device) at positions p0 .. p0+count-1 through every layer as one batch
// (no head: qwen.c discards the logits of prompt positions), writing their KV-cache rows exactly as the decode
// step would. Enqueued on the model's stream; 0, or -1 after set_error().
static int prefill_batch(Model &m, const int *tokens, int p0, int count) {
    const Config &c = m.c;
    const int dim = c.dim, hid = c.hidden_dim, kv = m.kv_dim, L = c.n_layers, nmax = dim > hid ? dim : hid;
    Model::Batch &b = m.pf;
    cudaError_t e = cudaSuccess;
    if (!b.cap) {
        const int cap = m.ctx < kBatchCap ? m.ctx : kBatchCap, ldx = (cap + 3) / 4 * 4;
        if ((e = cudaMalloc(&b.x, (size_t)cap * dim * 4)) != cudaSuccess ||
            (e = cudaMalloc(&b.qkv, (size_t)cap * (dim + 2 * kv) * 4)) != cudaSuccess ||
            (e = cudaMalloc(&b.qb, (size_t)cap * dim * 4)) != cudaSuccess ||
            (e = cudaMalloc(&b.att, (size_t)cap * dim * 4)) != cudaSuccess ||
            (e = cudaMalloc(&b.out, (size_t)cap * dim * 4)) != cudaSuccess ||
            (e = cudaMalloc(&b.h1, (size_t)cap * hid * 4)) != cudaSuccess ||
            (e = cudaMalloc(&b.h3, (size_t)cap * hid * 4)) != cudaSuccess ||
            (e = cudaMalloc(&b.xs, (size_t)(nmax / 32) * ldx * 4)) != cudaSuccess ||
            (e = cudaMalloc(&b.xq, (size_t)cap * nmax)) != cudaSuccess ||
            (e = cudaFuncSetAttribute(attention_rows_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)attention_rows_smem_bytes<64>(kMaxCtx, kVChunk))) != cudaSuccess ||
            (e = cudaFuncSetAttribute(attention_gqa_rows_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      kGqaSmemMax)) != cudaSuccess ||
            (e = cudaStreamCreateWithFlags(&b.side[0], cudaStreamNonBlocking)) != cudaSuccess ||
            (e = cudaStreamCreateWithFlags(&b.side[1], cudaStreamNonBlocking)) != cudaSuccess ||
            (e = cudaEventCreateWithFlags(&b.fork, cudaEventDisableTiming)) != cudaSuccess ||
            (e = cudaEventCreateWithFlags(&b.join[0], cudaEventDisableTiming)) != cudaSuccess ||
            (e = cudaEventCreateWithFlags(&b.join[1], cudaEventDisableTiming)) != cudaSuccess) {
            set_error("mvb_qwen_prefill: batch buffers: %s", cudaGetErrorString(e));
            return -1;
        }
        b.cap = cap;
    }
    if (count < 1 || count > b.cap || p0 < 0 || p0 + count > m.ctx) {
        set_error("mvb_qwen_prefill: batch of %d tokens at %d outside the buffers", count, p0);
        return -1;
    }
    const cudaStream_t s = m.stream;
    const int ldx = (count + 3) / 4 * 4, T = kThreads;
    auto gemm = [&](const Mat &w, int n, int d, float *out, int ldo, cudaStream_t st) {
        return gemm_launch(w.w, w.s, b.xq, b.xs, out, n, d, count, ldx, ldo, 4, st);
    };
    // the side streams start after everything queued on the model's stream so far (fork) and the model's stream
    // goes on after both (join): matmuls of the same input, writing disjoint outputs, run side by side
    auto fork = [&]() {
        return cudaEventRecord(b.fork, s) != cudaSuccess || cudaStreamWaitEvent(b.side[0], b.fork, 0) != cudaSuccess ||
               cudaStreamWaitEvent(b.side[1], b.fork, 0) != cudaSuccess;
    };
    auto join = [&]() {
        for (int i = 0; i < 2; i++)
            if (cudaEventRecord(b.join[i], b.side[i]) != cudaSuccess || cudaStreamWaitEvent(s, b.join[i], 0) != cudaSuccess)
                return true;
        return false;
    };
    embed_rows_kernel<<<count, T, 0, s>>>((const int8_t *)m.emb.w, (const uint16_t *)m.emb.s, tokens, b.x, dim);
    for (int l = 0; l < L; l++) {
        // the previous layer's down residual (x += its matmul output) is folded into this norm
        norm_quant_rows_kernel<<<count, T, 2 * dim * 4, s>>>(b.x, l > 0 ? b.out : nullptr, m.attn_norm + (size_t)l * dim,
                                                             c.rms_eps, dim, b.xq, b.xs, ldx);
        const int ldq = dim + 2 * kv;
        if (fork() || gemm(m.wq[l], dim, dim, b.qkv, ldq, s) || gemm(m.wk[l], dim, kv, b.qkv + dim, ldq, b.side[0]) ||
            gemm(m.wv[l], dim, kv, b.qkv + dim + kv, ldq, b.side[1]) || join())
            return -1;
        rope_cache_rows_kernel<<<count, T, 0, s>>>(b.qkv, ldq, m.bq + (size_t)l * dim, m.bk + (size_t)l * kv,
                                                   m.bv + (size_t)l * kv, m.rope, m.kcache + (size_t)l * m.ctx * kv,
                                                   m.vcache + (size_t)l * m.ctx * kv, b.qb, p0, dim, kv, m.hs);
        // shared memory for the positions this batch reaches only: more CTAs per SM. Where the kv head's keys and
        // values of every position fit in one CTA's shared memory, one CTA per (token, kv head) stages them once
        // for the group's query heads; otherwise one CTA per (token, query head) reads them in chunks.
        const int npos = p0 + count, kv_mul = c.n_heads / c.n_kv_heads;
        const size_t gqa_smem = attention_gqa_smem_bytes<64>(npos, kv_mul);
        if (gqa_smem <= (size_t)kGqaSmemMax && kv_mul * 32 <= 1024) {
            // quantizes its outputs for the o projection itself
            attention_gqa_rows_kernel<64><<<dim3(count, c.n_kv_heads), kv_mul * 32, gqa_smem, s>>>(
                b.qb, m.kcache + (size_t)l * m.ctx * kv, m.vcache + (size_t)l * m.ctx * kv, b.xq, b.xs, ldx, p0, dim,
                kv, kv_mul, npos, m.et);
        } else {
            const int vchunk = npos < kVChunk ? (npos + 7) / 8 * 8 : kVChunk;
            attention_rows_kernel<64><<<dim3(count, c.n_heads), T, attention_rows_smem_bytes<64>(npos, vchunk), s>>>(
                b.qb, m.kcache + (size_t)l * m.ctx * kv, m.vcache + (size_t)l * m.ctx * kv, b.att, p0, dim, kv,
                kv_mul, npos, vchunk, m.et);
            quant_rows_kernel<<<count, T, dim * 4, s>>>(b.att, dim, b.xq, b.xs, ldx);
        }
        if (gemm(m.wo[l], dim, dim, b.out, dim, s)) return -1;
        // x += the o matmul's output, then the FFN norm, in one kernel
        norm_quant_rows_kernel<<<count, T, 2 * dim * 4, s>>>(b.x, b.out, m.ffn_norm + (size_t)l * dim, c.rms_eps, dim,
                                                             b.xq, b.xs, ldx);
        if (fork() || gemm(m.w1[l], dim, hid, b.h1, hid, s) || gemm(m.w3[l], dim, hid, b.h3, hid, b.side[0]) ||
            join())
            return -1;
        swiglu_quant_rows_kernel<<<dim3(count, (hid / 32 + 31) / 32), T, 0, s>>>(b.h1, b.h3, hid, m.et, b.xq, b.xs,
                                                                                 ldx);
        if (gemm(m.w2[l], hid, dim, b.out, dim, s)) return -1;
        // x += the down matmul's output: here after the last layer, else in the next layer's first norm
        if (l == L - 1) residual_rows_kernel<<<(count * dim + T - 1) / T, T, 0, s>>>(b.x, b.out, (size_t)count * dim);
    }
    if ((e = cudaGetLastError()) != cudaSuccess) {
        set_error("mvb_qwen_prefill: launch failed: %s", cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

}  // namespace decode
}  // namespace mvb

using namespace mvb;
using namespace mvb::decode;

namespace mvb {
namespace decode {

// Captures one forward step into m->graph, then the instrumented copy (events between kernels, no programmatic
// overlap) into m->prof_graph and the stamped copy (the step as it runs, every kernel stamping the global timer)
// into m->stamp_graph, replacing any earlier capture. Nothing of the model may be in flight.
static cudaError_t capture_graphs(Model *m) {
    cudaError_t e;
    if (m->graph) cudaGraphExecDestroy(m->graph);
    if (m->prof_graph) cudaGraphExecDestroy(m->prof_graph);
    if (m->stamp_graph) cudaGraphExecDestroy(m->stamp_graph);
    m->graph = m->prof_graph = m->stamp_graph = nullptr;
    for (cudaEvent_t ev : m->prof_ev) cudaEventDestroy(ev);
    m->prof_ev.clear();
    m->info.clear();
    for (int pass = 0; pass < 3; pass++) {
        cudaGraph_t graph;
        int count = 0;
        const bool pdl = m->pdl;
        if (pass == 1) {
            m->pdl = false;
            m->prof_ev.resize(m->kernels_per_step + 1);
            for (auto &ev : m->prof_ev)
                if ((e = cudaEventCreate(&ev)) != cudaSuccess) return e;
        }
        m->stamping = pass == 2;
        if ((e = cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal)) != cudaSuccess) return e;
        cudaError_t le = pass == 0 ? enqueue_step(*m, &count, nullptr, &m->info)
                                   : enqueue_step(*m, &count, pass == 1 ? m->prof_ev.data() : nullptr, nullptr);
        e = cudaStreamEndCapture(m->stream, &graph);
        m->pdl = pdl;
        m->stamping = false;
        if (le != cudaSuccess) return le;
        if (e != cudaSuccess) return e;
        e = cudaGraphInstantiate(pass == 0 ? &m->graph : (pass == 1 ? &m->prof_graph : &m->stamp_graph), graph, 0);
        cudaGraphDestroy(graph);
        if (e != cudaSuccess) return e;
        if (pass == 0) m->kernels_per_step = count;
    }
    return cudaSuccess;
}

// The second half of loading, common to both families: with the config, the weight pointers and the RoPE table
// (ctx * hs floats) in place, allocates the activations, caches and state, and captures the step graphs.
// Returns m, or null after set_error() (m is freed).
static Model *finish_load(Model *m, const std::vector<float> &rope, const char *who) {
    const Config &c = m->c;
    const int dim = c.dim, kv = m->kv_dim, hid = c.hidden_dim, L = c.n_layers;
    cudaError_t e = cudaSuccess;
    auto fail = [&](const char *what) -> Model * {
        set_error("%s: %s: %s", who, what, cudaGetErrorString(e));
        destroy(m);
        return nullptr;
    };
    const size_t kvbytes = (size_t)L * m->ctx * kv * 4;
    if ((e = cudaMalloc(&m->x, dim * 4)) != cudaSuccess || (e = cudaMalloc(&m->xb, dim * 4)) != cudaSuccess ||
        (e = cudaMalloc(&m->qkv, (dim + 2 * kv) * 4)) != cudaSuccess ||
        (e = cudaMalloc(&m->hb, (size_t)hid * 4)) != cudaSuccess ||
        (e = cudaMalloc(&m->logits, (size_t)c.vocab_size * 4)) != cudaSuccess ||  // room for a full head
        (e = cudaMalloc(&m->kcache, kvbytes)) != cudaSuccess || (e = cudaMalloc(&m->vcache, kvbytes)) != cudaSuccess ||
        (e = cudaMalloc(&m->rope, rope.size() * 4)) != cudaSuccess ||
        (e = cudaMalloc(&m->xq_n, dim)) != cudaSuccess || (e = cudaMalloc(&m->xs_n, dim / 32 * 4)) != cudaSuccess ||
        (e = cudaMalloc(&m->counters, (size_t)(5 * L + 2) * 4)) != cudaSuccess ||
        (e = cudaMalloc(&m->prompt, (size_t)m->ctx * 4)) != cudaSuccess ||
        (e = cudaMalloc(&m->ids, (size_t)m->ctx * 4)) != cudaSuccess ||
        (e = cudaMalloc(&m->st, sizeof(State))) != cudaSuccess ||
        (e = cudaMalloc(&m->stamps, (size_t)(5 * L + 2) * 2 * sizeof(unsigned long long))) != cudaSuccess)
        return fail("buffers");
    if ((e = cudaMemcpy(m->rope, rope.data(), rope.size() * 4, cudaMemcpyHostToDevice)) != cudaSuccess ||
        (e = cudaMemset(m->kcache, 0, kvbytes)) != cudaSuccess ||
        (e = cudaMemset(m->vcache, 0, kvbytes)) != cudaSuccess ||
        (e = cudaMemset(m->st, 0, sizeof(State))) != cudaSuccess ||
        (e = cudaMemset(m->counters, 0, (size_t)(5 * L + 2) * 4)) != cudaSuccess ||
        (e = set_attention_smem_all()) != cudaSuccess)
        return fail("init");
    if ((e = cudaHostAlloc(&m->ring, sizeof(State) * Model::kRing, cudaHostAllocDefault)) != cudaSuccess)
        return fail("pinned state");
    m->et = expf_table_device();
    if (!m->et.slots) {
        e = cudaErrorUnknown;
        return fail("expf table");
    }
    if ((e = capture_graphs(m)) != cudaSuccess) return fail("capture");
    return m;
}

// Device, stream and PDL setting of a new model. 0, or -1 after set_error().
static int open_device(Model *m, const char *who) {
    cudaError_t e = cudaGetDevice(&m->device);
    if (const char *pd = getenv("MVB_PDL")) m->pdl = atoi(pd) != 0;
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        set_error("%s: %s", who, cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

// Maps a whole file read-only (for the file loaders: the weights go from the page cache straight to HBM).
struct FileMap {
    void *p = nullptr;
    size_t n = 0;
    explicit FileMap(const char *path) {
        const int fd = path ? open(path, O_RDONLY) : -1;
        if (fd < 0) return;
        struct stat st;
        if (fstat(fd, &st) == 0 && st.st_size > 0) {
            void *q = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
            if (q != MAP_FAILED) {
                p = q;
                n = (size_t)st.st_size;
            }
        }
        close(fd);
    }
    ~FileMap() {
        if (p) munmap(p, n);
    }
};

}  // namespace decode
}  // namespace mvb

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
    m->family = kQwen;
    memcpy(&m->c, b + 8, sizeof(Config));
    Config &c = m->c;
    // qwen.c:223-228's checks, plus this implementation's own limits
    if (c.group_size != 32 || c.emb_bits != 8 || c.n_heads <= 0 || c.n_kv_heads <= 0 || c.dim % c.n_heads ||
        c.n_heads % c.n_kv_heads || (c.dim / c.n_heads) % 2 || c.dim % 128 || c.hidden_dim % 128 ||
        (c.dim / c.n_heads * c.n_kv_heads) % 16 || c.dim > kMaxDim || c.hidden_dim > kMaxN || c.dim / c.n_heads != 64 ||
        c.head_k <= 0 || c.vocab_size <= 0 || c.n_layers <= 0) {
        set_error("mvb_qwen_load: unsupported config (group %d, embedding %d-bit, dim %d, hidden %d, heads %d/%d; "
                  "this decode needs head size 64, dim <= %d, hidden <= %d)", c.group_size, c.emb_bits, c.dim,
                  c.hidden_dim, c.n_heads, c.n_kv_heads, kMaxDim, kMaxN);
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
    if (open_device(m, "mvb_qwen_load")) {
        destroy(m);
        return nullptr;
    }
    cudaError_t e;
    if ((e = cudaMalloc(&m->image, bytes)) != cudaSuccess ||
        (e = cudaMemcpy(m->image, image, bytes, cudaMemcpyHostToDevice)) != cudaSuccess) {
        set_error("mvb_qwen_load: weights: %s", cudaGetErrorString(e));
        destroy(m);
        return nullptr;
    }
    m->image_bytes = bytes;
    auto at = [&](size_t o) { return m->image + o; };
    m->attn_norm = (const float *)at(o_attn); m->ffn_norm = (const float *)at(o_ffn);
    m->bq = (const float *)at(o_bq); m->bk = (const float *)at(o_bk); m->bv = (const float *)at(o_bv);
    m->out_norm = (const float *)at(o_norm); m->head_ids = (const int32_t *)at(o_ids);
    auto conv = [&](const std::vector<MatOff> &v, std::vector<Mat> &dst) {
        for (auto &x : v) dst.push_back(Mat{at(x.w), at(x.s)});
    };
    conv(q, m->wq); conv(k, m->wk); conv(vv, m->wv); conv(o, m->wo); conv(g, m->w1); conv(dn, m->w2); conv(u, m->w3);
    m->head = m->head_trim = Mat{at(hd[0].w), at(hd[0].s)};
    m->ids_trim = m->head_ids;
    m->head_rows = c.head_k;
    m->emb = Mat{at(em[0].w), at(em[0].s)};
    // RoPE table, exactly qwen.c:504-508 per position
    std::vector<float> rope((size_t)m->ctx * m->hs);
    for (int pos = 0; pos < m->ctx; pos++)
        for (int i = 0; i < m->hs / 2; i++) {
            double a = pos * pow(c.rope_theta, -2.0 * i / m->hs);
            rope[(size_t)pos * m->hs + i] = (float)cos(a);
            rope[(size_t)pos * m->hs + m->hs / 2 + i] = (float)sin(a);
        }
    return finish_load(m, rope, "mvb_qwen_load");
}

extern "C" void *mvb_qwen_load_file(const char *path, int ctx) {
    clear_error();
    FileMap f(path);
    if (!f.p) {
        set_error("mvb_qwen_load_file: cannot map %s", path ? path : "(null)");
        return nullptr;
    }
    return mvb_qwen_load(f.p, f.n, ctx);
}

// runq v2 checkpoint (runq.c:318-357): 256-byte header, fp32 rmsnorm weights, then int8 values each followed by
// their fp32 group scales (runq.c:274-289) for the embedding, wq, wk, wv, wo, w1, w2, w3 (per layer) and, unless it
// is shared with the embedding, the classifier (runq.c:291-316). The file's tensors follow one another with no
// padding; here each is copied into its own 256-byte-aligned slot of one device allocation (the kernels read
// weights 16 bytes at a time), straight from the caller's bytes: no host copy is made.
extern "C" void *mvb_runq_load(const void *image, size_t bytes, int ctx) {
    clear_error();
    const uint8_t *b = static_cast<const uint8_t *>(image);
    uint32_t magic = 0;
    int32_t version = 0;
    if (b && bytes >= 256) {
        memcpy(&magic, b, 4);
        memcpy(&version, b + 4, 4);
    }
    if (!b || bytes < 256 || magic != 0x616b3432 || version != 2) {  // runq.c:322-329
        set_error("mvb_runq_load: not a runq version 2 checkpoint");
        return nullptr;
    }
    int32_t h[7];  // dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len (runq.c:28-36)
    memcpy(h, b + 8, sizeof h);
    const uint8_t shared = b[36];
    int32_t gs;
    memcpy(&gs, b + 37, 4);
    Model *m = new Model;
    m->family = kRunq;
    Config &c = m->c;
    c = Config{};
    c.dim = h[0]; c.hidden_dim = h[1]; c.n_layers = h[2]; c.n_heads = h[3]; c.n_kv_heads = h[4];
    c.vocab_size = h[5]; c.max_seq_len = h[6]; c.group_size = gs; c.emb_bits = 8;
    c.head_k = c.vocab_size;  // the classifier has a row per token
    c.rope_theta = 10000.0f;  // runq.c:509
    c.rms_eps = 1e-5f;        // runq.c:401
    const int hs = c.n_heads > 0 ? c.dim / c.n_heads : 0;
    // runq.c's FPGA build accepts group size 32 or 64 (runq.c:339-341; tools/bin2q80.py picks 64 when dim allows,
    // else 32); head sizes 32, 48 (stories15M) and 64 (stories110M)
    if ((gs != 32 && gs != 64) || c.n_heads <= 0 || c.n_kv_heads <= 0 || c.dim % c.n_heads ||
        c.n_heads % c.n_kv_heads || (hs != 32 && hs != 48 && hs != 64) || c.dim % gs || c.hidden_dim % gs ||
        c.dim > kMaxDim || c.hidden_dim > kMaxN || c.vocab_size <= 0 || c.n_layers <= 0 || c.max_seq_len <= 0) {
        set_error("mvb_runq_load: unsupported config (group %d, dim %d, hidden %d, heads %d/%d; this decode needs "
                  "group size 32 or 64 dividing dim and hidden, head size 32, 48 or 64, dim <= %d, hidden <= %d)",
                  gs, c.dim, c.hidden_dim, c.n_heads, c.n_kv_heads, kMaxDim, kMaxN);
        delete m;
        return nullptr;
    }
    m->hs = hs;
    m->kv_dim = hs * c.n_kv_heads;
    m->ctx = ctx < c.max_seq_len ? ctx : c.max_seq_len;
    if (m->ctx < 2 || m->ctx > kMaxCtx) {
        set_error("mvb_runq_load: context %d outside [2, %d]", m->ctx, kMaxCtx);
        delete m;
        return nullptr;
    }
    // the file's tensors in order (source offset, bytes) and their slots in the device arena
    const int L = c.n_layers, dim = c.dim, kv = m->kv_dim, hid = c.hidden_dim;
    struct Piece { size_t src, bytes, dst; };
    std::vector<Piece> pieces;
    size_t src = 256, dst = 0;
    auto piece = [&](size_t n) {
        pieces.push_back(Piece{src, n, dst});
        src += n;
        dst += (n + 255) & ~(size_t)255;
        return pieces.size() - 1;
    };
    const size_t p_att = piece((size_t)L * dim * 4), p_ffn = piece((size_t)L * dim * 4), p_fin = piece((size_t)dim * 4);
    struct MatPiece { size_t q, s; };
    auto mats = [&](int count, size_t d, size_t n) {
        std::vector<MatPiece> v(count);
        for (auto &x : v) {
            x.q = piece(d * n);
            x.s = piece(d * n / gs * 4);
        }
        return v;
    };
    auto em = mats(1, c.vocab_size, dim);
    auto q = mats(L, dim, dim), k = mats(L, kv, dim), vv = mats(L, kv, dim), o = mats(L, dim, dim),
         w1 = mats(L, hid, dim), w2 = mats(L, dim, hid), w3 = mats(L, hid, dim);
    auto cls = shared ? em : mats(1, c.vocab_size, dim);
    if (src > bytes) {
        set_error("mvb_runq_load: checkpoint is %zu bytes, but its header describes %zu", bytes, src);
        delete m;
        return nullptr;
    }
    if (open_device(m, "mvb_runq_load")) {
        destroy(m);
        return nullptr;
    }
    cudaError_t e = cudaMalloc(&m->image, dst);
    for (size_t i = 0; e == cudaSuccess && i < pieces.size(); i++)
        e = cudaMemcpy(m->image + pieces[i].dst, b + pieces[i].src, pieces[i].bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        set_error("mvb_runq_load: weights: %s", cudaGetErrorString(e));
        destroy(m);
        return nullptr;
    }
    m->image_bytes = dst;
    auto at = [&](size_t i) { return m->image + pieces[i].dst; };
    m->attn_norm = (const float *)at(p_att);
    m->ffn_norm = (const float *)at(p_ffn);
    m->out_norm = (const float *)at(p_fin);
    auto conv = [&](const std::vector<MatPiece> &v, std::vector<Mat> &out) {
        for (auto &x : v) out.push_back(Mat{at(x.q), at(x.s)});
    };
    conv(q, m->wq); conv(k, m->wk); conv(vv, m->wv); conv(o, m->wo); conv(w1, m->w1); conv(w2, m->w2); conv(w3, m->w3);
    m->emb = Mat{at(em[0].q), at(em[0].s)};
    m->head = Mat{at(cls[0].q), at(cls[0].s)};
    m->head_rows = c.vocab_size;
    // RoPE table per position, computed as runq.c:506-512 does it (float powf/cosf/sinf of the host C library);
    // pair j of a head is (2j, 2j + 1), whose head_dim is 2j
    std::vector<float> rope((size_t)m->ctx * hs);
    for (int pos = 0; pos < m->ctx; pos++)
        for (int j = 0; j < hs / 2; j++) {
            const int head_dim = 2 * j;
            const float freq = 1.0f / powf(10000.0f, head_dim / (float)hs);
            const float val = pos * freq;
            rope[(size_t)pos * hs + j] = cosf(val);
            rope[(size_t)pos * hs + hs / 2 + j] = sinf(val);
        }
    return finish_load(m, rope, "mvb_runq_load");
}

extern "C" void *mvb_runq_load_file(const char *path, int ctx) {
    clear_error();
    FileMap f(path);
    if (!f.p) {
        set_error("mvb_runq_load_file: cannot map %s", path ? path : "(null)");
        return nullptr;
    }
    return mvb_runq_load(f.p, f.n, ctx);
}

extern "C" void mvb_qwen_free(void *model) { destroy(static_cast<Model *>(model)); }

extern "C" int mvb_qwen_config(void *model, int *out) {
    Model *m = static_cast<Model *>(model);
    if (!m || !out) return -1;
    const Config &c = m->c;
    const int v[] = {c.dim, c.hidden_dim, c.n_layers, c.n_heads, c.n_kv_heads, c.vocab_size, m->head_rows, m->ctx,
                     m->kernels_per_step};
    memcpy(out, v, sizeof v);
    return 0;
}

// Switches a .qwb model's head between the file's trimmed head (head_k rows, ids through head_ids; qwen.c's) and
// the full vocabulary: Qwen2 ties the output head to the token embedding (gguf2qwb.py takes the trimmed head's
// rows from it), so the Q8 embedding serves as a vocab_size-row head whose argmax row is the token id. Recaptures
// the step graphs; the KV cache and state are kept. 0, or -1.
extern "C" int mvb_qwen_full_head(void *model, int on) {
    Model *m = static_cast<Model *>(model);
    if (!m) return -1;
    if (m->family == kRunq) {  // runq.c's classifier already has a row per token
        if (on) return 0;
        set_error("mvb_qwen_full_head: a runq model has no trimmed head");
        return -1;
    }
    if (wait_stream(*m, "mvb_qwen_full_head", timeout_s())) return -1;
    m->head = on ? m->emb : m->head_trim;
    m->head_ids = on ? nullptr : m->ids_trim;
    m->head_rows = on ? m->c.vocab_size : m->c.head_k;
    const cudaError_t e = capture_graphs(m);
    if (e != cudaSuccess) {
        set_error("mvb_qwen_full_head: capture: %s", cudaGetErrorString(e));
        return -1;
    }
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
    if (logits && cudaMemcpyAsync(logits, m->logits, (size_t)m->head_rows * 4, cudaMemcpyDeviceToHost, m->stream) !=
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

static int check_prompt(Model *m, const int *prompt, int n, const char *who) {
    if (!m || !prompt || n < 1 || n >= m->ctx) {
        set_error("%s: need 1 <= n < ctx", who);
        return -1;
    }
    for (int i = 0; i < n; i++)
        if (prompt[i] < 0 || prompt[i] >= m->c.vocab_size) {
            set_error("%s: token id %d out of range", who, prompt[i]);
            return -1;
        }
    if (cudaMemcpyAsync(m->prompt, prompt, (size_t)n * 4, cudaMemcpyHostToDevice, m->stream) != cudaSuccess) {
        set_error("%s: prompt upload failed", who);
        return -1;
    }
    return 0;
}

// The same state reached one decode step per fed token (the reference's own order of work).
extern "C" int mvb_qwen_prefill_tokenwise(void *model, const int *prompt, int n) {
    Model *m = static_cast<Model *>(model);
    if (check_prompt(m, prompt, n, "mvb_qwen_prefill_tokenwise")) return -1;
    if (set_state(*m, prompt[0], 0, n) || mvb_qwen_launch(m, n - 1)) return -1;
    return wait_stream(*m, "mvb_qwen_prefill_tokenwise", timeout_s() + 0.01 * n);
}

// Feeds prompt[0 .. n-2] (positions 0 .. n-2), leaving prompt[n-1] as the token of position n-1: the state
// qwen.c's (and runq.c's) generate() is in just before its first sampled token. For a .qwb model the fed tokens go
// through the layers in batches (tensor-core matmuls), writing the same KV-cache rows one decode step per token
// would; a runq model takes one decode step per token.
extern "C" int mvb_qwen_prefill(void *model, const int *prompt, int n) {
    Model *m = static_cast<Model *>(model);
    if (m && m->family == kRunq) return mvb_qwen_prefill_tokenwise(model, prompt, n);
    if (check_prompt(m, prompt, n, "mvb_qwen_prefill")) return -1;
    for (int p0 = 0; p0 < n - 1; p0 += kBatchCap)
        if (prefill_batch(*m, m->prompt + p0, p0, (n - 1 - p0) < kBatchCap ? n - 1 - p0 : kBatchCap)) return -1;
    if (set_state(*m, prompt[n - 1], n - 1, n)) return -1;
    if (wait_stream(*m, "mvb_qwen_prefill", timeout_s() + 0.01 * n)) return -1;
    const int st = mvb_gemm_status(m->stream);
    if (st) {
        set_error("mvb_qwen_prefill: a matmul wait gave up (code %d)", st);
        return -1;
    }
    return 0;
}

// Copies the KV cache rows of positions 0 .. positions-1 of every layer to k and v (host, n_layers * positions *
// kv_dim floats each, layer-major). 0, or -1.
extern "C" int mvb_qwen_cache(void *model, int positions, float *k, float *v) {
    Model *m = static_cast<Model *>(model);
    if (!m || !k || !v || positions < 1 || positions > m->ctx) return -1;
    const size_t row = (size_t)positions * m->kv_dim * 4;
    for (int l = 0; l < m->c.n_layers; l++) {
        const size_t off = (size_t)l * m->ctx * m->kv_dim;
        if (cudaMemcpyAsync(k + (size_t)l * positions * m->kv_dim, m->kcache + off, row, cudaMemcpyDeviceToHost,
                            m->stream) != cudaSuccess ||
            cudaMemcpyAsync(v + (size_t)l * positions * m->kv_dim, m->vcache + off, row, cudaMemcpyDeviceToHost,
                            m->stream) != cudaSuccess)
            return -1;
    }
    return wait_stream(*m, "mvb_qwen_cache", timeout_s());
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

// Runs the stamped copy of the step once from the current state (which it advances like a normal step) and writes,
// for every kernel k, us[2k] = when its first CTA got past its wait for kernel k - 1 and us[2k + 1] = when its last
// CTA finished, in microseconds after the first kernel's start. Returns the kernel count, or -1.
extern "C" int mvb_qwen_stamps(void *model, double *us, int cap) {
    Model *m = static_cast<Model *>(model);
    if (!m || !us || cap < 2 * m->kernels_per_step) return -1;
    const size_t bytes = (size_t)m->kernels_per_step * 2 * sizeof(unsigned long long);
    std::vector<unsigned long long> t(2 * (size_t)m->kernels_per_step);
    cudaError_t e = cudaMemsetAsync(m->stamps, 0, bytes, m->stream);
    if (e == cudaSuccess) e = cudaGraphLaunch(m->stamp_graph, m->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(t.data(), m->stamps, bytes, cudaMemcpyDeviceToHost, m->stream);
    if (e != cudaSuccess) {
        set_error("mvb_qwen_stamps: %s", cudaGetErrorString(e));
        return -1;
    }
    if (wait_stream(*m, "mvb_qwen_stamps", timeout_s())) return -1;
    const unsigned long long t0 = ~t[0];
    for (int k = 0; k < m->kernels_per_step; k++) {
        us[2 * k] = (double)(long long)(~t[2 * k] - t0) * 1e-3;
        us[2 * k + 1] = (double)(long long)(t[2 * k + 1] - t0) * 1e-3;
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

// qwen.c generate() at temperature 0 (qwen.c:669-712) for a .qwb model, runq.c generate() at temperature 0
// (runq.c:982-1026) for a runq model: the prompt fed (mvb_qwen_prefill), then greedy tokens until `steps` are
// generated, a stop token is sampled (<|im_end|> or <|endoftext|> for qwen.c, BOS = 1 for runq.c, runq.c:1016), or
// the context is full. Returns the count, stop token excluded.
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
        if (m->family == kRunq ? ids[i] == 1 : (ids[i] == kImEnd || ids[i] == kEndOfText)) return i;
    return n;
}

extern "C" int mvb_runq_generate(void *model, const int *prompt, int n_prompt, int steps, int *ids) {
    return mvb_qwen_generate(model, prompt, n_prompt, steps, ids);
}

// ---------------------------------------------------------------------------------------------------------------
// The decode's head path without any device allocation: final rmsnorm + quantize (norm_quant_kernel) into a
// scratch that lives in a file-scope device array, then the head matvec reading it. For callers that cannot
// allocate device memory (see mvb_norm_matvec4_static in include/matvec_b200.h).
namespace mvb {
namespace decode {

constexpr int kStaticNormMatvecMaxN = kMaxDim;  // 2048 columns
// n int8 quantized activations at offset 0, their n/32 fp32 scales at offset kStaticNormMatvecMaxN
static __device__ __align__(256) uint8_t g_norm_matvec_scratch[kStaticNormMatvecMaxN + kStaticNormMatvecMaxN / 32 * 4];

static std::mutex g_scratch_mu;
// device address of the array in each CUDA context it was looked up in, keyed by the context's unique ID
// (cuCtxGetId: never reused within a process, so the context a cudaDeviceReset() makes next gets a lookup of its own)
static std::map<unsigned long long, uint8_t *> g_scratch_addr;

// The array's device address in the current device's context, looked up once per context (in practice once per
// device: every runtime call of a device uses its one primary context). Host code only has a stand-in for the
// array's name; handing that to a kernel would read the wrong memory. Without a context ID (no driver entry
// points), the address is looked up on every call, which allocates nothing either.
static uint8_t *scratch_address(int dev) {
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    unsigned long long id = current_context_id();
    if (id) {
        auto it = g_scratch_addr.find(id);
        if (it != g_scratch_addr.end()) return it->second;
    }
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_norm_matvec_scratch);
    if (e != cudaSuccess || !p) {
        set_error("mvb_norm_matvec4_static: cannot get the scratch address on device %d: %s", dev,
                  cudaGetErrorString(e));
        return nullptr;
    }
    if (!id) id = current_context_id();  // the lookup made the device's context current if it was not yet
    if (id) g_scratch_addr[id] = static_cast<uint8_t *>(p);
    return static_cast<uint8_t *>(p);
}

}  // namespace decode
}  // namespace mvb

extern "C" int mvb_norm_matvec4_static(const float *x, const float *norm_w, float eps, const void *w, const void *ws,
                                       float *out, int n, int d, int wbits, void *stream) {
    using namespace mvb::decode;
    // every argument is checked before anything is launched: a refused call leaves the shared scratch (which a
    // call on another stream may be reading) and the output untouched
    if (!x || !norm_w || !w || !ws || !out) {
        set_error("mvb_norm_matvec4_static: null pointer argument");
        return -1;
    }
    if (((uintptr_t)x & 3) || ((uintptr_t)norm_w & 3) || ((uintptr_t)w & 15) || ((uintptr_t)ws & 1) ||
        ((uintptr_t)out & 3)) {
        set_error("mvb_norm_matvec4_static: misaligned pointer (w needs 16 bytes, ws 2, x, norm_w and out 4)");
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
