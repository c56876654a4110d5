// Batched prefill matmul on the 5th-generation tensor cores: M tokens at once through one quantized matrix.
//
// The reference prefills its prompt one token at a time through fpga_matvec4 (qwen.c:674-681); this computes
// the same M matvecs as one GEMM, out[m][i] = matvec of token m against row i, bit-identical to the reference
// C path for every token (qwen.c:436-456):
//     isum_g = sum_{k<32} w[i, 32g+k] * xq[m, 32g+k]               int32, exact
//     out    = ((0 + fl(fl(isum_0 * ws[i,0]) * xs[m,0])) + ...)    fp32, groups in order
// One group of 32 is exactly one K=32 step of tcgen05.mma.kind::i8, so the tensor cores produce each group's
// int32 sum for a 128-row x BN-token tile into tensor memory, and the epilogue warps apply the two rounded
// scale multiplies and the in-order add per group in fp32 registers.
//
// Tile = 128 weight rows x BN tokens; K is walked in blocks of 128 bytes (4 groups) through a ring of 4
// shared-memory stages. When the tiles exceed one wave and one CTA fills an SM, the grid is one CTA per SM and each
// CTA walks tiles blockIdx.x, + gridDim.x, ... (row tiles fastest) with one running k-block count, so the ring, the
// tensor-memory slots and their barrier phases carry on from one tile into the next: the next tile's copies and
// MMAs run under this tile's epilogue, and the per-CTA setup and teardown happen once. Otherwise one CTA per tile.
// Warp roles (320 threads; 448 for int4 weights):
//   warp 0   TMA producer (one thread): per k-block the weight tile (int8, or packed int4), the token tile
//            (both 128-byte swizzled, the layout the MMA descriptors describe) and the tokens' scales of the
//            block's four groups ([4][BN] fp32) into the next stage.
//   warp 1   allocates tensor memory; one thread issues the MMAs: per k-block, D[slot][k] = A_k x B_k^T for its
//            four groups into one of kSlots TMEM slots (4 for BN <= 32, else 2) of four BN-column group buffers,
//            then one commit. MMAs run asynchronously, up to kSlots - 1 k-blocks ahead of the epilogue.
//   warps 2-9  epilogue: two warps per TMEM lane quadrant (row = lane), each owning BN/2 token columns. Per
//            k-block: tcgen05.ld of the groups' int32 sums, release the slot and the stage, then per group and column
//            acc += fl(fl((float)isum * ws) * xs). (float)isum * ws is one fma on a biased integer: with
//            v = bits(isum + 0x4B400000) = 12582912 + isum (exact for |isum| < 2^22), fma(v, ws, -12582912 * ws)
//            rounds (v - 12582912) * ws = isum * ws once, and -12582912 * ws is exact because ws has at most 11
//            significant bits (an fp16 value).
//   warps 10-13  int4 weights only: unpack each stage's packed tile into its int8 operand tile (same swizzle) as
//            soon as its copies land, eight 16-byte chunks per thread, for the MMA. The tile holds 16 * v (the
//            nibble in the high half of its byte), so the group sums are 16 * isum, |16 * isum| <= 16 * 32 * 8 * 128
//            < 2^22, and the epilogue's fma above takes ws / 16. Done by the epilogue warps,
//            the unpack sits on their per-k-block path: 896 x 4864 at 128 tokens takes 41.4 us that way, 31.9 us
//            with these warps.
// The token tile BN (16, 32 or 64) is the largest that keeps row tiles x token tiles at half the SM count or more:
// the in-order sum over groups rules out splitting K across CTAs.
// Every mbarrier wait is bounded (kGemmWaitNs of %globaltimer); a wait that runs out records an error, the
// roles stop, outstanding copies and MMAs are waited for (bounded), tensor memory is freed and the kernel ends.
// No TMA multicast; no clusters.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <mutex>

#include "../../include/matvec_b200.h"
#include "matvec_kernels.cuh"
#include "mvb_runtime.h"

namespace mvb {
namespace gemm {

constexpr int kBM = 128;          // weight rows per CTA (MMA M)
constexpr int kBK = 128;          // int8 K bytes per stage (4 groups)
constexpr int kThreads = 320;   // producer, MMA and 8 epilogue warps
constexpr int kEpiWarps = 8;
constexpr int kUnpackWarps = 4;  // int4 weights: 4 more warps unpack each stage's packed tile
template <int BITS>
constexpr int threads_of() { return BITS == 4 ? kThreads + kUnpackWarps * 32 : kThreads; }
constexpr unsigned long long kGemmWaitNs = 1000000000ull;

// error codes in the error word (first failure wins)
enum : int { kErrNone = 0, kErrFullWait = 1, kErrEmptyWait = 2, kErrTmemFull = 3, kErrTmemEmpty = 4, kErrRaw = 5 };

__device__ int g_gemm_error;

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ unsigned long long now_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Waits for the phase with the given parity to complete; false after kGemmWaitNs (the error is recorded).
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int err) {
    const uint32_t a = smem_u32(bar);
    unsigned long long t0 = 0;
    for (uint32_t i = 0;; i++) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(a), "r"(parity)
            : "memory");
        if (done) return true;
        if ((i & 1023) == 1023) {
            const unsigned long long t = now_ns();
            if (!t0) t0 = t;
            else if (t - t0 > kGemmWaitNs) {
                atomicCAS(&g_gemm_error, kErrNone, err);
                return false;
            }
        }
    }
}

__device__ __forceinline__ bool failed() { return *(volatile int *)&g_gemm_error != kErrNone; }

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

// Shared-memory matrix descriptor of a K-major operand tile in the 128-byte swizzled canonical layout: rows of 128
// bytes, 8-row atoms of 1024 bytes one after another (stride byte offset 1024), leading byte offset 16 (unused for
// this layout), descriptor version 1, layout type 2 (SWIZZLE_128B). Field positions as in the sm100 descriptor
// definition (start >> 4 in bits 0-13, LBO >> 4 in 16-29, SBO >> 4 in 32-45, version in 46-47, layout in 61-63).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) |
           ((uint64_t)2 << 61);
}

// Instruction descriptor of tcgen05.mma.kind::i8: D s32 (bits 4-5 = 2), A and B signed int8 (bits 7-9, 10-12 =
// 1), both K-major, N >> 3 in bits 17-22, M >> 4 in bits 24-28.
__host__ __device__ constexpr uint32_t idesc_i8(int m, int n) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(0)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 8 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, int (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// int4 nibbles of one 32-bit word (8 two's complement elements v, element 2i in the low nibble of byte i) -> the
// 8 int8 values 16 * v as two words in element order: a nibble moved into the high half of its byte is the int8
// 16 * v, sign included (two logic operations and two byte permutes per word, no sign extension). The MMA's group
// sums are then 16 * isum, and the epilogue's weight scale ws / 16.
__device__ __forceinline__ uint2 unpack_int4_x16(uint32_t w) {
    const uint32_t lo = (w << 4) & 0xF0F0F0F0u, hi = w & 0xF0F0F0F0u;
    return make_uint2(__byte_perm(lo, hi, 0x5140), __byte_perm(lo, hi, 0x7362));
}

struct GemmParams {
    const uint16_t *ws;  // d x ng fp16 weight scales
    const float *xs;     // ng x ldx fp32 token scales, group-major
    float *out;          // m rows of ldo fp32 (the first d used), token-major
    int n, d, m, ldx, ng, ldo;
    PeerTargets peers;   // GATHER: the gathered outputs and the completion counters
};

__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// N consecutive 32-bit TMEM columns (N = 8, 16 or 32) of this thread's lane.
template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, int (&r)[N]) {
    if constexpr (N == 8) {
        tmem_ld8(taddr, r);
    } else if constexpr (N == 16) {
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
            "%15}, [%16];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
              "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
            : "r"(taddr));
    } else {
        static_assert(N == 32, "8, 16 or 32 columns");
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
            "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
              "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
              "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
              "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
            : "r"(taddr));
    }
}

// One shared-memory stage: the int8 weight tile, the token tile, the packed int4 weight tile (int4 only) and the
// tokens' scales of the k-block's four groups ([4][BN] fp32).
template <int BN, int BITS>
struct Smem {
    static constexpr int kA = kBM * kBK;                        // int8 operand tile (1024-aligned)
    static constexpr int kB = BN * kBK;                         // token tile (1024-aligned)
    static constexpr int kRaw = BITS == 4 ? kBM * kBK / 2 : 0;  // packed int4 tile
    static constexpr int kX = 4 * BN * 4;                       // token scales
    static constexpr int kStage = (kA + kB + kRaw + kX + 1023) / 1024 * 1024;
    // four stages (measured: six to eight, which fit in shared memory, were slower: fewer resident CTAs; for int4
    // weights, one 448-thread CTA per SM, six to eight were no faster)
    static constexpr int kStages = 4;
    static constexpr size_t kNatural = (size_t)kStages * kStage + 1024 /* align */ + 256 /* barriers */;
    // TMEM: kSlots k-block slots of four group buffers of BN columns (four slots where they fit, so the MMAs can
    // run up to three k-blocks ahead of the epilogue). The shared memory request is raised so that no more CTAs
    // than an SM's 512 columns hold can be resident (an allocation never has to wait).
    static constexpr int kSlots = BN <= 32 ? 4 : 2;
    static constexpr int kCols = kSlots * 4 * BN < 32 ? 32 : kSlots * 4 * BN;
    static constexpr size_t kFloor = 233472 / (512 / kCols + 1) + 1024;
    static constexpr size_t kBytes = kNatural > kFloor ? kNatural : kFloor;
    static_assert(kCols <= 512 && kBytes <= 232448, "tensor memory or shared memory per CTA");
};

// Unpacks the packed int4 tile of a stage ([128 rows][64 bytes]) into its int8 operand tile ([128 rows][128 bytes],
// 16-byte chunk c of row r stored at chunk c ^ (r & 7): the 128-byte swizzle the TMA applies to the int8 tiles).
// Values 16 * v (unpack_int4_x16). Shared by the NT threads of the calling warps (thread index i): thread i does
// chunk i & 7 of rows i / 8, + NT / 8, ... (NT / 8 is a multiple of 8, so the swizzled chunk stays the thread's).
// Ends with the proxy fence that makes the generic-proxy writes visible to the MMA.
template <int NT>
__device__ __forceinline__ void unpack_tile(const uint8_t *raw, uint8_t *a, int i) {
    static_assert(NT % 64 == 0 && (kBM * 8) % NT == 0, "whole passes of rows in steps of 8");
    const int r = i >> 3, c = i & 7;
    const uint8_t *src = raw + r * (kBK / 2) + c * 8;
    uint8_t *dst = a + (r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4);
#pragma unroll
    for (int k = 0; k < kBM * 8 / NT; k++) {
        const uint2 pk = *reinterpret_cast<const uint2 *>(src + k * (NT / 8) * (kBK / 2));
        const uint2 e0 = unpack_int4_x16(pk.x), e1 = unpack_int4_x16(pk.y);
        *reinterpret_cast<uint4 *>(dst + k * (NT / 64) * 1024) = make_uint4(e0.x, e0.y, e1.x, e1.y);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ONE: every CTA has exactly one tile (the grid is the tile count, within one wave), so the tile loops fold away.
template <int BN, int BITS, bool GATHER, bool ONE>
__global__ void __launch_bounds__(threads_of<BITS>(), 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                const __grid_constant__ CUtensorMap map_x, const GemmParams p) {
    using S = Smem<BN, BITS>;
    constexpr int kStages = S::kStages;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // aligned to 1024 bytes by an offset added to the shared array itself: a pointer that went through an integer
    // cast would be generic, and every stage access through it a generic load or store
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + (size_t)kStages * S::kStage);
    // full: the stage's copies landed. ready: its int4 tile is unpacked (4 unpack warps). empty: the epilogue
    // has finished the stage's k-block (8 warps; its MMAs had completed before that). tfull / tempty: a TMEM
    // k-block slot was written (one commit) / has been read (8 warps).
    constexpr int kSlots = S::kSlots;
    uint64_t *full = bar, *ready = bar + kStages, *empty = bar + 2 * kStages, *tfull = bar + 3 * kStages,
             *tempty = tfull + kSlots;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tempty + kSlots);
    constexpr int kCols = S::kCols;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nkb = (p.n + kBK - 1) / kBK;
    const int ngroups = p.ng;
    // this CTA's tiles: t = blockIdx.x, + gridDim.x, ...; tile t is row tile t % nrow, token tile t / nrow (the
    // order of a two-dimensional grid of row tiles by token tiles)
    const int nrow = (p.d + kBM - 1) / kBM;
    const int ntiles = nrow * ((p.m + BN - 1) / BN);
    const int mine = ONE ? 1 : ntiles > (int)blockIdx.x ? (ntiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    auto tile_of = [&](int i) { return (int)blockIdx.x + i * (int)gridDim.x; };

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&ready[s], kUnpackWarps);
            mbar_init(&empty[s], kEpiWarps);
        }
        for (int j = 0; j < kSlots; j++) {
            mbar_init(&tfull[j], 1);
            mbar_init(&tempty[j], kEpiWarps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    auto stage_a = [&](int s) { return smem + (size_t)s * S::kStage; };
    auto stage_b = [&](int s) { return smem + (size_t)s * S::kStage + S::kA; };
    auto stage_raw = [&](int s) { return smem + (size_t)s * S::kStage + S::kA + S::kB; };
    auto stage_x = [&](int s) { return reinterpret_cast<float *>(smem + (size_t)s * S::kStage + S::kA + S::kB + S::kRaw); };
    constexpr uint32_t kTx = (BITS == 4 ? kBM * kBK / 2 : kBM * kBK) + BN * kBK + 4 * BN * 4;

    if (warp == 0) {
        // ---------------- producer: one thread issues the copies of each stage ----------------
        if (lane == 0) {
            int j = 0;  // this CTA's k-blocks issued so far (stage j % kStages, phase j / kStages)
            bool stop = false;
            for (int i = 0; i < mine && !stop; i++) {
                const int t = tile_of(i);
                const int row0 = (t % nrow) * kBM, m0 = (t / nrow) * BN;
                for (int kb = 0; kb < nkb; kb++) {
                    const int s = j % kStages;
                    if (j >= kStages && !mbar_wait(&empty[s], ((j / kStages) - 1) & 1, kErrEmptyWait)) {
                        stop = true;
                        break;
                    }
                    mbar_expect_tx(&full[s], kTx);
                    if (BITS == 4) tma_load_2d(stage_raw(s), &map_a, &full[s], kb * (kBK / 2), row0);
                    else tma_load_2d(stage_a(s), &map_a, &full[s], kb * kBK, row0);
                    tma_load_2d(stage_b(s), &map_b, &full[s], kb * kBK, m0);
                    tma_load_2d(stage_x(s), &map_x, &full[s], m0, kb * (kBK / 32));
                    j++;
                }
            }
            // copies still in flight land before the CTA can end: wait (bounded) for the last phase of each stage
            for (int jj = j > kStages ? j - kStages : 0; jj < j; jj++)
                mbar_wait(&full[jj % kStages], (jj / kStages) & 1, kErrFullWait);
        }
    } else if (warp == 1) {
        // ---------------- MMA issue: one thread ----------------
        if (lane == 0) {
            const uint32_t idesc = idesc_i8(kBM, BN);
            int j = 0;  // this CTA's k-blocks issued so far (TMEM slot j % kSlots)
            bool stop = false;
            for (int i = 0; i < mine && !stop; i++) {
                for (int kb = 0; kb < nkb; kb++) {
                    const int s = j % kStages, slot = j % kSlots;
                    if (!mbar_wait(&full[s], (j / kStages) & 1, kErrFullWait) ||
                        (BITS == 4 && !mbar_wait(&ready[s], (j / kStages) & 1, kErrRaw)) ||
                        // the slot's previous k-block must have been read by the epilogue
                        (j >= kSlots && !mbar_wait(&tempty[slot], ((j / kSlots) - 1) & 1, kErrTmemEmpty))) {
                        stop = true;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(stage_a(s)), b0 = smem_u32(stage_b(s));
                    const int ng_kb = min(kBK / 32, ngroups - kb * (kBK / 32));
                    for (int k = 0; k < ng_kb; k++)
                        mma_i8(tmem + (slot * 4 + k) * BN, smem_desc(a0 + 32 * k), smem_desc(b0 + 32 * k), idesc);
                    mma_commit(&tfull[slot]);
                    j++;
                }
            }
            // all MMAs complete before tensor memory is freed: wait (bounded) for the last commit
            if (j > 0) mbar_wait(&tfull[(j - 1) % kSlots], ((j - 1) / kSlots) & 1, kErrTmemFull);
        }
    } else if (warp < 2 + kEpiWarps) {
        // ---------------- epilogue ----------------
        constexpr int kCw = BN / 2;               // columns per thread
        constexpr int kLd = kCw < 32 ? kCw : 32;  // columns per TMEM load
        const int q = warp & 3, half = (warp - 2) >> 2;
        const int col0 = half * kCw;
        // this rank's completed calls: the output buffer of this call (parity) in every rank's gather
        const unsigned call = GATHER ? *p.peers.calls : 0u;
        bool ok = true;
        // this thread's row of tile i, and its weight scales (row 0's past the last row)
        auto row_of = [&](int i) { return (tile_of(i) % nrow) * kBM + q * 32 + lane; };
        auto scales_of = [&](int row) { return p.ws + (size_t)(row < p.d ? row : 0) * p.ng; };
        uint16_t wnext[4];  // the scales of the next k-block, loaded one k-block ahead (across tiles too)
        if (mine > 0) {
            const uint16_t *w0 = scales_of(row_of(0));
#pragma unroll
            for (int k = 0; k < 4; k++) wnext[k] = k < ngroups ? __ldg(w0 + k) : (uint16_t)0;
        }
        int j = 0;  // this CTA's k-blocks consumed so far
        for (int i = 0; i < mine && ok; i++) {
            const int t = tile_of(i);
            const int row = row_of(i), m0 = (t / nrow) * BN;
            float acc[kCw];
#pragma unroll
            for (int c = 0; c < kCw; c++) acc[c] = 0.0f;
            const uint16_t *wsr = scales_of(row);
            const uint16_t *wsn = i + 1 < mine ? scales_of(row_of(i + 1)) : wsr;
            for (int kb = 0; kb < nkb; kb++, j++) {
                const int s = j % kStages, slot = j % kSlots;
                uint16_t wcur[4];
                const bool last = kb + 1 == nkb;
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    wcur[k] = wnext[k];
                    // the next k-block's scales: this row's, or after the last k-block the next tile's first four
                    const int g = last ? k : (kb + 1) * 4 + k;
                    wnext[k] = g < ngroups ? __ldg((last ? wsn : wsr) + g) : (uint16_t)0;
                }
                if (!(ok = mbar_wait(&full[s], (j / kStages) & 1, kErrFullWait))) break;  // this stage's token scales
                if (!(ok = mbar_wait(&tfull[slot], (j / kSlots) & 1, kErrTmemFull))) break;
                tc_fence_after();
                const float *xst = stage_x(s);
                const int ng_kb = min(kBK / 32, ngroups - kb * (kBK / 32));
                // the block's group sums are read kG groups per TMEM round trip (all four when they fit in registers)
                constexpr int kG = kCw <= 16 ? 4 : 2;
#pragma unroll
                for (int k0 = 0; k0 < 4; k0 += kG) {
                    if (k0 >= ng_kb) break;
                    int isum[kG][kCw / kLd][kLd];
#pragma unroll
                    for (int g = 0; g < kG; g++)
#pragma unroll
                        for (int ch = 0; ch < kCw / kLd; ch++)
                            tmem_ld<kLd>(tmem + ((uint32_t)(q * 32) << 16) + (slot * 4 + k0 + g) * BN + col0 + ch * kLd,
                                         isum[g][ch]);
                    tmem_wait_ld();
#pragma unroll
                    for (int g = 0; g < kG; g++) {
                        const int k = k0 + g;
                        if (k >= ng_kb) break;
                        // int4 tiles hold 16 * v: their sums are 16 * isum, and ws / 16 is exact (a power of two)
                        const float wsc = BITS == 4 ? __fmul_rn(scale_from_f16(wcur[k]), 0.0625f) : scale_from_f16(wcur[k]);
                        const float ncw = __fmul_rn(-12582912.0f, wsc);  // exact: wsc has <= 11 significant bits
                        const float *xsg = xst + k * BN + col0;
#pragma unroll
                        for (int c = 0; c < kCw; c += 4) {
                            const float4 x4 = *reinterpret_cast<const float4 *>(xsg + c);  // same address in every lane
                            const float xv[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
                            for (int i4 = 0; i4 < 4; i4++) {
                                const float v = __int_as_float(isum[g][(c + i4) / kLd][(c + i4) % kLd] + 0x4B400000);
                                const float pw = __fmaf_rn(v, wsc, ncw);  // fl(isum * ws)
                                acc[c + i4] = __fadd_rn(acc[c + i4], __fmul_rn(pw, xv[i4]));
                            }
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&tempty[slot]);
                    mbar_arrive(&empty[s]);
                }
            }
            if (!ok || failed() || row >= p.d) continue;
            if (!GATHER) {
#pragma unroll
                for (int c = 0; c < kCw; c++)
                    if (m0 + col0 + c < p.m) p.out[(size_t)(m0 + col0 + c) * p.ldo + row] = acc[c];
            } else {
                // every rank's gathered output: 32 lanes store 32 consecutive rows of one token (NVLink for peers)
#pragma unroll
                for (int c = 0; c < kCw; c++)
                    if (m0 + col0 + c < p.m) {
                        const size_t o = (size_t)(m0 + col0 + c) * p.ldo + p.peers.col0 + row;
#pragma unroll
                        for (int r = 0; r < kMaxGatherRanks; r++)
                            if (r < p.peers.world) p.peers.out[r][(call & 1) * p.peers.obuf + o] = acc[c];
                    }
            }
        }
        if (GATHER && p.peers.world > 1) fence_acq_rel_gpu();  // this thread's stores, before the CTA is counted
    } else if (BITS == 4) {
        // ---------------- int4 unpack warps ----------------
        // Per k-block, the packed weight tile into its int8 operand tile, for the MMA: off the epilogue warps' path,
        // as far ahead as the ring holds stages. The stage was refilled only after the epilogue had finished the
        // k-block before it (whose MMAs had completed).
        const int ut = threadIdx.x - kThreads;  // 0 .. 127
        for (int j = 0; j < mine * nkb; j++) {
            const int s = j % kStages;
            if (!mbar_wait(&full[s], (j / kStages) & 1, kErrRaw)) break;
            unpack_tile<kUnpackWarps * 32>(stage_raw(s), stage_a(s), ut);
            __syncwarp();
            if (lane == 0) mbar_arrive(&ready[s]);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols) : "memory");
    if (GATHER && threadIdx.x == 0 && atomicAdd(p.peers.done, 1u) == gridDim.x - 1) {
        // the last CTA of this rank: every CTA's rows are stored. Signal every rank (one system-scope fence, then
        // relaxed adds: a release), then wait, bounded, until every rank has signalled this call (the last read an
        // acquire load). With one rank the end of the kernel publishes the rows: only the call counter advances.
        *p.peers.done = 0;
        const unsigned call = *p.peers.calls;
        const unsigned target = (call + 1u) * (unsigned)p.peers.world;  // every rank's signal of this call
        if (p.peers.world > 1) {
            fence_acq_rel_sys();
            for (int r = 0; r < kMaxGatherRanks; r++)
                if (r < p.peers.world)
                    asm volatile("red.relaxed.sys.global.add.u32 [%0], 1;" ::"l"(p.peers.arrive[r]) : "memory");
            const unsigned long long t0 = now_ns();
            for (uint32_t i = 0;; i++) {
                unsigned v;
                asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p.peers.arrive[p.peers.rank])
                             : "memory");
                if ((int)(v - target) >= 0) {
                    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p.peers.arrive[p.peers.rank])
                                 : "memory");
                    break;
                }
                if ((i & 63) == 63 && now_ns() - t0 > 2 * kGemmWaitNs) {
                    atomicExch(p.peers.err, 1);
                    break;
                }
            }
        }
        *p.peers.calls = call + 1u;  // every other CTA read the old value before it was counted
    }
}

// ---------------------------------------------------------------------------------------------------------------
// host side: tensor maps through the driver entry point (no link against the driver library)

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static std::once_flag once;
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    std::call_once(once, [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    });
    return fn;
}

// 2-D tensor map over rows x cols elements (row pitch cols elements), box box_rows x box_cols, optional 128B
// swizzle; uint8 or fp32 elements.
static bool make_map(CUtensorMap *map, const void *base, uint64_t cols, uint64_t rows, uint32_t box_cols,
                     uint32_t box_rows, bool swizzle, bool fp32 = false) {
    auto fn = encode_fn();
    if (!fn) return false;
    const uint64_t esz = fp32 ? 4 : 1;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * esz};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, fp32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base),
              dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// CTAs of `kernel` (blocks of `threads`, smem bytes of dynamic shared memory, cols TMEM columns) that one SM holds, from
// its registers, its shared memory and its tensor-memory columns, times the SMs. (The runtime's occupancy query
// answers one CTA per SM for the 16-token tiles that hold two, as ncu's launch statistics and the waves of a launch
// show.) Cached per device and kernel.
static int gemm_slots(const void *kernel, size_t smem, int cols, int threads) {
    static std::mutex mu;
    static std::map<std::pair<int, const void *>, int> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    std::lock_guard<std::mutex> lock(mu);
    const auto key = std::make_pair(dev, kernel);
    const auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    cudaFuncAttributes fa = {};
    int sms = 0, regs_sm = 0, smem_sm = 0, reserved = 0, threads_sm = 0;
    if (cudaFuncGetAttributes(&fa, kernel) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&regs_sm, cudaDevAttrMaxRegistersPerMultiprocessor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&threads_sm, cudaDevAttrMaxThreadsPerMultiProcessor, dev) != cudaSuccess || sms <= 0) {
        cudaGetLastError();
        return 148;
    }
    const int warps = threads / 32;
    const int regs_warp = (fa.numRegs * 32 + 255) / 256 * 256;  // registers are given to a warp 256 at a time
    int per = regs_warp > 0 ? regs_sm / regs_warp / warps : 1;
    per = std::min(per, (int)(smem_sm / (smem + fa.sharedSizeBytes + reserved)));
    per = std::min(per, threads_sm / threads);
    per = std::min(per, 512 / cols);
    return cache[key] = sms * std::max(per, 1);
}

template <int BN, int BITS>
static cudaError_t launch_gemm(const CUtensorMap &ma, const CUtensorMap &mb, const CUtensorMap &mx, const GemmParams &p,
                               cudaStream_t s, bool gather) {
    const size_t smem = Smem<BN, BITS>::kBytes;
    // persistent: at most one CTA per SM, each walking its tiles (the fixed per-CTA costs -- barrier setup, tensor
    // memory, the pipeline's first copies, the gather's fence and count -- paid once per SM). A grid of one wave,
    // or a tile size with two or more CTAs per SM, runs the one-tile form, one CTA per tile: with two CTAs per SM
    // a static split leaves some SMs a tile more than the hardware's own scheduling of the waves does (65536 x
    // 896 at 16 tokens: 22.5 against 19.1 us).
    const int tiles = ((p.d + kBM - 1) / kBM) * ((p.m + BN - 1) / BN);
    auto multi = gather ? gemm_kernel<BN, BITS, true, false> : gemm_kernel<BN, BITS, false, false>;
    auto single = gather ? gemm_kernel<BN, BITS, true, true> : gemm_kernel<BN, BITS, false, true>;
    // both forms may take the shared memory, and prefer the largest shared-memory carveout
    cudaError_t e = cudaSuccess;
    for (auto k : {multi, single}) {
        if (e == cudaSuccess) e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    }
    if (e != cudaSuccess) return e;
    const int slots = gemm_slots((const void *)multi, smem, Smem<BN, BITS>::kCols, threads_of<BITS>());
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const bool one = tiles <= slots || slots >= 2 * sms;
    if (one) single<<<tiles, threads_of<BITS>(), smem, s>>>(ma, mb, mx, p);
    else multi<<<slots, threads_of<BITS>(), smem, s>>>(ma, mb, mx, p);
    return cudaGetLastError();
}

}  // namespace gemm
}  // namespace mvb

using namespace mvb;
using namespace mvb::gemm;

namespace mvb {

int gemm_launch(const void *w, const void *ws, const void *xq, const float *xs, float *out, int n, int d, int m, int ldx,
                int ldo, int wbits, cudaStream_t stream, const PeerTargets *peers) {
    if (wbits != 4 && wbits != 8) {
        set_error("mvb_gemm4: unsupported wbits=%d (need 4 or 8)", wbits);
        return -1;
    }
    if (n <= 0 || n % 32 || n > kMaxN || d <= 0 || m <= 0 || ldx < m || ldx % 4 || ldo < d) {
        set_error("mvb_gemm4: unsupported n=%d d=%d m=%d ldx=%d (need n %% 32 == 0, n <= %d, d, m >= 1, ldx >= m, "
                  "ldx %% 4 == 0)", n, d, m, ldx, kMaxN);
        return -1;
    }
    if (!w || !ws || !xq || !xs || (!out && !peers) || ((uintptr_t)w & 15) || ((uintptr_t)xq & 15) || ((uintptr_t)ws & 1) ||
        ((uintptr_t)xs & 15) || ((uintptr_t)out & 3)) {
        set_error("mvb_gemm4: null or misaligned pointer (w and xq 16 bytes, xs 16, ws 2, out 4)");
        return -1;
    }
    using namespace gemm;
    CUtensorMap ma, mb, mx;
    const bool ok_a = wbits == 4 ? make_map(&ma, w, (uint64_t)n / 2, (uint64_t)d, kBK / 2, kBM, false)
                                 : make_map(&ma, w, (uint64_t)n, (uint64_t)d, kBK, kBM, true);
    // token tile: the largest of 64, 32, 16 that still gives at least half as many CTAs as SMs, else 16 (measured
    // on the config-4 shapes at 128 and 512 tokens: larger tiles win while the grid stays that wide, e.g. 4864 x
    // 896 at 128 tokens in 15.1 us with 64 against 20.2 with 32; narrow matrices want the most CTAs)
    const int row_tiles = (d + kBM - 1) / kBM;
    int bn = 16;
    for (int c : {64, 32}) {
        if (c < 2 * m && (long)row_tiles * ((m + c - 1) / c) >= 72) {
            bn = c;
            break;
        }
    }
    const bool ok_b = make_map(&mb, xq, (uint64_t)n, (uint64_t)m, kBK, bn, true);
    // token scales, group-major: box of 4 groups x bn tokens
    const bool ok_x = make_map(&mx, xs, (uint64_t)ldx, (uint64_t)(n / 32), bn, kBK / 32, false, true);
    if (!ok_a || !ok_b || !ok_x) {
        set_error("mvb_gemm4: cannot build the TMA descriptors (driver entry point missing or bad layout)");
        return -1;
    }
    GemmParams p;
    p.ws = static_cast<const uint16_t *>(ws);
    p.xs = xs;
    p.out = out;
    p.n = n;
    p.d = d;
    p.m = m;
    p.ldx = ldx;
    p.ng = n / 32;
    p.ldo = ldo;
    p.peers = peers ? *peers : PeerTargets{};
    const bool g = peers != nullptr;
    cudaError_t e;
    if (wbits == 4) {
        e = bn == 16 ? launch_gemm<16, 4>(ma, mb, mx, p, stream, g)
          : bn == 32 ? launch_gemm<32, 4>(ma, mb, mx, p, stream, g) : launch_gemm<64, 4>(ma, mb, mx, p, stream, g);
    } else {
        e = bn == 16 ? launch_gemm<16, 8>(ma, mb, mx, p, stream, g)
          : bn == 32 ? launch_gemm<32, 8>(ma, mb, mx, p, stream, g) : launch_gemm<64, 8>(ma, mb, mx, p, stream, g);
    }
    if (e != cudaSuccess) {
        set_error("mvb_gemm4: launch failed: %s", cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

}  // namespace mvb

extern "C" int mvb_gemm4(const void *w, const void *ws, const void *xq, const float *xs, float *out, int n, int d, int m,
                         int ldx, int wbits, void *stream) {
    return gemm_launch(w, ws, xq, xs, out, n, d, m, ldx, d, wbits, static_cast<cudaStream_t>(stream));
}

// Synchronizes `stream` and returns (and clears) the device error word of the GEMM kernels: 0, or the code of the
// first wait that ran out; -1 if the stream itself failed.
extern "C" int mvb_gemm_status(void *stream) {
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (cudaStreamSynchronize(s) != cudaSuccess) return -1;
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_gemm_error, sizeof v) != cudaSuccess) return -1;
    if (v) {
        const int z = 0;
        cudaMemcpyToSymbol(g_gemm_error, &z, sizeof z);
    }
    return v;
}
