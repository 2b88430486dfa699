// Prompt / verification projections on the 5th-generation tensor cores.
//
// Y[t][r] = sum_k W[r][k] * X[t][k] with W the exact BF16 weights and X the FP32
// activations. X is split once into BF16 terms hi = bf16(x), mid = bf16(x - hi),
// lo = bf16(x - hi - mid), and every K step issues one tcgen05.mma per term into
// the same FP32 accumulator in tensor memory. Products of BF16 pairs are exact
// in FP32, so three terms carry x to about 24 significant bits, FP32 class.
// Two terms (16 bits) were measured against three on B200: projections stay
// within 1e-5 relative L2 (2.5e-6 against 6.5e-7) and the 455-token 8B prefill
// is 13 % faster (gate_up 311 against 370 us), but the whole model drifts -
// prefill logits 1.7e-3 from the oracle, 3.3 times the spread of two valid FP32
// summation orders - and its 64 greedy tokens no longer match the oracle's,
// so three terms stay (kTcTerms). Replaces the reference's FP32 batched matvec
// (src/matmul*.s, runtime/kernels.metal:299-365).
//
// The tensor cores truncate while they accumulate, so error grows with the
// number of MMAs chained into one accumulator. Each 64-wide K block therefore
// gets a fresh accumulator (a ring of 2..16 in TMEM, see tc_acc_count) and the epilogue
// warps fold every block into FP32 registers with round-to-nearest adds: no
// tensor-core chain is longer than one block, whatever K is.
//
// Tiling ("swap AB"): the weight rows are the M = 128 operand, tokens are N.
// One CTA computes one 128 x N tile:
//   warp 0      TMA producer: W tile [128 x 64] and hi/lo tiles [N x 64] per
//               stage, 128-byte swizzle, no multicast;
//   warp 1      allocates the TMEM accumulator; one lane issues the MMAs and
//               tcgen05.commit releases each stage / signals the epilogue;
//   warps 2-5   epilogue: tcgen05.ld of their TMEM lane quadrant, stores of
//               Y[token][row] (coalesced along rows).
// All waits are bounded; a timeout sets an error flag and the CTA drains.
//
// Split K (gridDim.z > 1, for a few tokens over few row tiles, e.g. the
// projections of a verification block or of a batch of decode requests): CTA
// z folds K blocks [z*kb/splits, (z+1)*kb/splits) and writes its partial tile
// to part[z]; splitk_sum_kernel adds the partials in z order, so the result
// does not depend on scheduling.
#pragma once
#include <cuda.h>

#include "common.cuh"
#include "../../include/plamo_synthetic.h"

namespace plamo {

constexpr int kTcM = 128;
constexpr int kTcK = 64;  // BF16 elements per stage row: 128 bytes, one swizzle atom
// Warps: TMA producer, MMA issuer, then the epilogue warps that fold every K
// block's accumulator into registers. A tile of 64 or more tokens gets two
// epilogue warps per TMEM lane quadrant, each folding half of the columns:
// with one, the fold (tcgen05.ld of 128 columns and 128 adds per K block)
// took longer than the block's three MMAs and held the tensor pipe at ~52 %.
template <int N>
__host__ __device__ constexpr int tc_epi_warps() {
    return N >= 64 ? 8 : 4;
}
template <int N>
__host__ __device__ constexpr int tc_threads() {
    return (2 + tc_epi_warps<N>()) * 32;
}
constexpr int kTcMaxStages = 10;
constexpr int kTcAccMax = 16;
// TMEM accumulators (one K block each) in a ring of 256 columns: with few
// tokens per tile a K block is quick to multiply, so the MMAs may run up to
// 16 blocks ahead of the epilogue's folds instead of stalling on it.
// TMEM columns between accumulators: a token-major tile's accumulators start
// on 32-column boundaries (the folds' 32-column loads stay aligned).
template <int N, bool TOKM = false>
__host__ __device__ constexpr int tc_acc_stride() {
    return TOKM ? (N + 31) / 32 * 32 : N;
}
// A token-major tile allocates all 512 columns (two accumulators of 192
// columns round up to it), so it keeps as many accumulators as they hold:
// two of 192 columns, three of 144 or 160. A 128-token weight-major tile
// keeps two in 256 columns: four (all 512) measured slower on the 8B
// down_proj (219 against 214 us), the next launch's CTAs then waiting for
// TMEM.
template <int N, bool TOKM = false>
__host__ __device__ constexpr int tc_acc_count() {
    return TOKM ? 512 / tc_acc_stride<N, true>() : N <= 16 ? 16 : N <= 32 ? 8 : N <= 64 ? 4 : 2;
}
// Columns folded by the first of a lane quadrant's two epilogue warps (the
// second takes the rest): a multiple of 32, so both start 32-aligned.
template <int N>
__host__ __device__ constexpr int tc_fold_split() {
    return tc_epi_warps<N>() == 8 ? 32 * (N / 64) : N;
}
constexpr int kTcTerms = 3;  // BF16 terms of each FP32 activation (2 or 3: loads and MMAs follow it)
static_assert(kTcTerms == 2 || kTcTerms == 3, "two or three BF16 terms");

struct TcGemmParams {
    float *y;  // [T][ys]
    uint64_t ys;
    uint32_t T, R, K;
    uint32_t *error;
    float *part;  // split K: [splits][T][R] partial tiles
    // Gate/up pairs (token-major tiles only, glu != nullptr): a tile's first
    // N/2 weight rows are gate rows [tile*N/2, +N/2) of map_w and the other
    // N/2 the same up rows of map_u; the epilogue writes the BF16 terms of
    // SwiGLU(gate, up) to glu ([3][T][glu_inter], planes glu_plane apart)
    // instead of Y.
    uint16_t *glu;
    uint64_t glu_plane;
    uint32_t glu_inter;
};

// ---- tcgen05 / TMA primitives ------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}
// K-major operand, 128-byte swizzle: 8-row atoms of 1024 bytes, rows 128 bytes apart.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((addr >> 4) & 0x3FFF);   // start address
    d |= static_cast<uint64_t>(1) << 16;                 // leading byte offset (unused for swizzled K-major)
    d |= static_cast<uint64_t>(1024 >> 4) << 32;         // stride byte offset: next 8-row atom
    d |= static_cast<uint64_t>(1) << 46;                 // descriptor version (sm_100)
    d |= static_cast<uint64_t>(2) << 61;                 // layout: 128-byte swizzle
    return d;
}
// kind::f16 instruction descriptor: BF16 x BF16 -> FP32, both K-major, M x N.
__host__ __device__ constexpr uint32_t tc_idesc(uint32_t m, uint32_t n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((n >> 3) << 17) | ((m >> 4) << 24);
}
__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// 32 consecutive FP32 accumulator columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 columns without the wait: several loads in flight, then one tmem_wait_ld().
__device__ __forceinline__ void tmem_ld32_async(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 16 consecutive FP32 accumulator columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// One pipeline stage: the A operand's 128 rows and the B operand's N rows of a
// 64-wide K block, three activation terms on the activation side.
inline size_t tc_stage_bytes(uint32_t n, bool tokm = false) {
    return tokm ? kTcTerms * static_cast<size_t>(kTcM) * 128 + 128ull * n
                : static_cast<size_t>(kTcM) * 128 + kTcTerms * 128ull * n;
}
inline size_t tc_smem_bytes(uint32_t n, int stages, bool tokm = false) {
    return stages * tc_stage_bytes(n, tokm) + 1024;
}
__host__ __device__ constexpr uint32_t tc_pow2_cols(uint32_t cols) {
    uint32_t p = 32;
    while (p < cols) p *= 2;
    return p;
}

// Everything an epilogue warp needs from its CTA.
struct TcEpilogue {
    TcGemmParams p;
    uint32_t tmem, warp, lane, kblocks;
    uint64_t *acc_full, *acc_empty;
    int *abort_flag;
    unsigned char *base;  // the stage buffers (the token-major store's staging tile)
    uint32_t row0, tok0;
};

// Add COUNT accumulator columns at taddr (32-aligned start) into sum.
template <int COUNT>
__device__ __forceinline__ void tc_fold_block(float (&sum)[COUNT], uint32_t taddr) {
    static_assert(COUNT % 16 == 0, "folds move 16 or 32 columns per load");
    if constexpr (COUNT % 64 == 0) {
        // Two loads in flight per wait.
#pragma unroll
        for (int c = 0; c < COUNT; c += 64) {
            uint32_t r0[32], r1[32];
            tmem_ld32_async(taddr + c, r0);
            tmem_ld32_async(taddr + c + 32, r1);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                sum[c + i] = __fadd_rn(sum[c + i], __uint_as_float(r0[i]));
                sum[c + 32 + i] = __fadd_rn(sum[c + 32 + i], __uint_as_float(r1[i]));
            }
        }
    } else {
        // One load per wait (96 or 80 columns: two in flight would spill).
        constexpr int C32 = COUNT / 32 * 32;
#pragma unroll
        for (int c = 0; c < C32; c += 32) {
            float v[32];
            tmem_ld32(taddr + c, v);
#pragma unroll
            for (int i = 0; i < 32; ++i) sum[c + i] = __fadd_rn(sum[c + i], v[i]);
        }
        if constexpr (COUNT > C32) {
            float v[16];
            tmem_ld16(taddr + C32, v);
#pragma unroll
            for (int i = 0; i < 16; ++i) sum[C32 + i] = __fadd_rn(sum[C32 + i], v[i]);
        }
    }
}

// Fold every K block's partial into FP32 registers (IEEE adds, in order) for
// this warp's TMEM lane quadrant, columns [COL0, COL0 + COUNT), then store
// them (or the split-K partial tile).
template <int N, bool TOKM, int COL0, int COUNT, int ACC, uint32_t STRIDE>
__device__ __forceinline__ void tc_fold_store(const TcEpilogue &e) {
    const TcGemmParams &p = e.p;
    const uint32_t quad = e.warp & 3;  // TMEM lanes this warp may access
    const uint32_t lanes = (quad * 32) << 16;
    float sum[COUNT];
#pragma unroll
    for (int i = 0; i < COUNT; ++i) sum[i] = 0.0f;
    bool ok = true;
    for (uint32_t kb = 0; kb < e.kblocks; ++kb) {
        const uint32_t a = kb % ACC;
        if (!mbar_wait(&e.acc_full[a], (kb / ACC) & 1u) || *reinterpret_cast<volatile int *>(e.abort_flag)) {
            ok = false;
            if (p.error && e.lane == 0) atomicExch(p.error, 3u);
            break;
        }
        tc_fence_after();
        tc_fold_block<COUNT>(sum, e.tmem + lanes + a * STRIDE + COL0);
        tc_fence_before();
        __syncwarp();
        if (e.lane == 0) mbar_arrive(&e.acc_empty[a]);
    }
    float *out = gridDim.z > 1 ? p.part + static_cast<uint64_t>(blockIdx.z) * p.T * p.R : p.y;
    const uint64_t stride = gridDim.z > 1 ? p.R : p.ys;
    if constexpr (TOKM) {
        // This lane is one token and its columns are consecutive weight
        // rows, so direct stores would scatter 32 output rows per
        // instruction. The tile goes through shared memory instead (the
        // stage buffers: every copy has landed and every MMA has read
        // them once the last block is folded), then each warp writes
        // whole token rows, 32 consecutive floats per instruction.
        constexpr uint32_t OS = N + 1;  // odd row stride: the column writes hit 32 banks
        float *tile = reinterpret_cast<float *>(e.base);
        const uint32_t tl = quad * 32 + e.lane;
#pragma unroll
        for (int j = 0; j < COUNT; ++j) tile[tl * OS + COL0 + j] = sum[j];
        asm volatile("bar.sync 1, %0;" ::"r"(tc_epi_warps<N>() * 32) : "memory");
        const uint32_t ew = e.warp - 2;
        if (p.glu) {
            // Columns [0, N/2) are gate rows, [N/2, N) the matching up rows:
            // SwiGLU, then its hi/mid/lo BF16 terms (the split of
            // split_hilo_kernel), 32 consecutive outputs per instruction.
            constexpr uint32_t HN = N / 2;
            const uint32_t j0 = blockIdx.y * HN;
            for (uint32_t r = ew; r < kTcM; r += tc_epi_warps<N>()) {
                const uint32_t t = e.tok0 + r;
                if (!ok || t >= p.T) continue;
                for (uint32_t c = e.lane; c < HN; c += 32) {
                    if (j0 + c >= p.glu_inter) continue;
                    const float v = swiglu(tile[r * OS + c], tile[r * OS + HN + c]);
                    const uint16_t h = plamo_bf16_round(v);
                    const float r1 = __fsub_rn(v, __uint_as_float(static_cast<uint32_t>(h) << 16));
                    const uint16_t md = plamo_bf16_round(r1);
                    const float r2 = __fsub_rn(r1, __uint_as_float(static_cast<uint32_t>(md) << 16));
                    const uint64_t i = static_cast<uint64_t>(t) * p.glu_inter + j0 + c;
                    p.glu[i] = h;
                    p.glu[p.glu_plane + i] = md;
                    p.glu[2 * p.glu_plane + i] = plamo_bf16_round(r2);
                }
            }
            return;
        }
        for (uint32_t r = ew; r < kTcM; r += tc_epi_warps<N>()) {
            const uint32_t t = e.tok0 + r;
            if (!ok || t >= p.T) continue;
            for (uint32_t c = e.lane; c < N; c += 32)
                if (e.row0 + c < p.R) out[static_cast<uint64_t>(t) * stride + e.row0 + c] = tile[r * OS + c];
        }
    } else {
        const uint32_t row = e.row0 + quad * 32 + e.lane;
        if (ok && row < p.R) {
#pragma unroll
            for (int j = 0; j < COUNT; ++j) {
                const uint32_t t = e.tok0 + COL0 + j;
                if (t < p.T) out[static_cast<uint64_t>(t) * stride + row] = sum[j];
            }
        }
    }
}

// Two tile layouts (TOKM):
//   weight-major (false): A = 128 weight rows, B = N tokens' terms; the
//     accumulator's TMEM lanes are weight rows, its columns tokens (N a
//     multiple of 16, <= 128). Suits few tokens.
//   token-major (true): A = 128 tokens' terms, B = N weight rows (N = 192):
//     lanes are tokens, columns weight rows; each K block then carries 1.5
//     times the MMA work of a 128 x 128 tile with 25 % fewer bytes per MMA,
//     and a 5120-row projection of 455 tokens is one wave of tiles.
template <int N, bool TOKM = false>
__global__ void __launch_bounds__(tc_threads<N>(), 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_u,
                   const __grid_constant__ CUtensorMap map_hi, const __grid_constant__ CUtensorMap map_mid,
                   const __grid_constant__ CUtensorMap map_lo, TcGemmParams p, int stages) {
    extern __shared__ __align__(128) unsigned char tc_smem_raw[];
    __shared__ __align__(8) uint64_t full_bar[kTcMaxStages];
    __shared__ __align__(8) uint64_t empty_bar[kTcMaxStages];
    constexpr int kTcAcc = tc_acc_count<N, TOKM>();
    __shared__ __align__(8) uint64_t acc_full[kTcAccMax];
    __shared__ __align__(8) uint64_t acc_empty[kTcAccMax];
    __shared__ uint32_t tmem_base;
    __shared__ int abort_flag;

    // 1024-byte aligned stage buffers (128-byte swizzle atoms).
    unsigned char *base = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const uint32_t stage_bytes = TOKM ? kTcTerms * kTcM * 128 + N * 128 : kTcM * 128 + kTcTerms * N * 128;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Token tiles run fastest: the CTAs that share one weight tile start
    // together, so it crosses HBM once and the others read it from L2.
    const uint32_t row0 = blockIdx.y * (TOKM ? N : kTcM), tok0 = blockIdx.x * (TOKM ? kTcM : N);
    const uint32_t kall = (p.K + kTcK - 1) / kTcK;
    const uint32_t kb0 = kall * blockIdx.z / gridDim.z;
    const uint32_t kblocks = kall * (blockIdx.z + 1) / gridDim.z - kb0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int a = 0; a < kTcAcc; ++a) {
            mbar_init(&acc_full[a], 1);
            mbar_init(&acc_empty[a], tc_epi_warps<N>());  // one arrival per epilogue warp
        }
        abort_flag = 0;
        fence_barrier_init();
        prefetch_tensormap(&map_w);
        if (TOKM && p.glu) prefetch_tensormap(&map_u);
        prefetch_tensormap(&map_hi);
        prefetch_tensormap(&map_mid);
        prefetch_tensormap(&map_lo);
    }
    constexpr uint32_t kStride = tc_acc_stride<N, TOKM>();
    constexpr uint32_t kCols = tc_pow2_cols(kTcAcc * kStride);  // power of two >= 32
    if (warp == 1) {  // the whole warp allocates the accumulators' TMEM columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                     "r"(kCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;
    pdl_launch_dependents();
    pdl_wait();

    if (warp == 0 && lane == 0) {
        uint32_t s = 0, phase = 0, issued = 0;
        for (uint32_t kb = 0; kb < kblocks; ++kb) {
            if (kb >= static_cast<uint32_t>(stages) && !mbar_wait(&empty_bar[s], phase ^ 1u)) {
                abort_flag = 1;
                if (p.error) atomicExch(p.error, 3u);
                break;
            }
            unsigned char *st = base + s * stage_bytes;
            mbar_expect_tx(&full_bar[s], stage_bytes);
            const int kx = static_cast<int>((kb0 + kb) * kTcK);
            // Stage layout: [A rows][B rows]; the activation side holds its
            // terms hi, mid(, lo) one after another.
            constexpr uint32_t wofs = TOKM ? kTcTerms * kTcM * 128 : 0;
            constexpr uint32_t tofs = TOKM ? 0 : kTcM * 128, tstep = (TOKM ? kTcM : N) * 128;
            if (TOKM && p.glu) {  // gate rows, then the same up rows
                const int g0 = static_cast<int>(blockIdx.y * (N / 2));
                tma_load_2d(st + wofs, &map_w, kx, g0, &full_bar[s]);
                tma_load_2d(st + wofs + (N / 2) * 128, &map_u, kx, g0, &full_bar[s]);
            } else {
                tma_load_2d(st + wofs, &map_w, kx, static_cast<int>(row0), &full_bar[s]);
            }
            tma_load_2d(st + tofs, &map_hi, kx, static_cast<int>(tok0), &full_bar[s]);
            tma_load_2d(st + tofs + tstep, &map_mid, kx, static_cast<int>(tok0), &full_bar[s]);
            if constexpr (kTcTerms == 3)
                tma_load_2d(st + tofs + 2 * tstep, &map_lo, kx, static_cast<int>(tok0), &full_bar[s]);
            issued = kb + 1;
            if (++s == static_cast<uint32_t>(stages)) {
                s = 0;
                phase ^= 1u;
            }
        }
        // Every copy issued has landed before the CTA can exit (immediate
        // when the MMAs consumed them; bounded otherwise).
        for (uint32_t k = issued > static_cast<uint32_t>(stages) ? issued - stages : 0; k < issued; ++k)
            mbar_wait(&full_bar[k % stages], (k / stages) & 1u);
    } else if (warp == 1 && lane == 0) {
        constexpr uint32_t idesc = tc_idesc(kTcM, N);
        uint32_t s = 0, phase = 0;
        for (uint32_t kb = 0; kb < kblocks; ++kb) {
            const uint32_t a = kb % kTcAcc;
            if (kb >= static_cast<uint32_t>(kTcAcc) &&
                !mbar_wait(&acc_empty[a], (kb / kTcAcc - 1) & 1u)) {  // epilogue drained it
                abort_flag = 1;
                if (p.error) atomicExch(p.error, 3u);
                break;
            }
            if (!mbar_wait(&full_bar[s], phase)) {
                abort_flag = 1;
                if (p.error) atomicExch(p.error, 3u);
                break;
            }
            tc_fence_after();
            const uint32_t sa = smem_u32(base + s * stage_bytes);
            const uint32_t acc = tmem + a * kStride;
            if constexpr (TOKM) {
                // A: the terms' [128 tokens] tiles; B: the weight tile.
                const uint32_t th = sa, tm = th + kTcM * 128, tl = tm + kTcM * 128;
                const uint32_t bw = sa + kTcTerms * kTcM * 128;
#pragma unroll
                for (int k = 0; k < kTcK / 16; ++k) {  // 16 BF16 = 32 bytes per MMA K step
                    const uint64_t db = smem_desc_sw128(bw + 32 * k);
                    tc_mma(acc, smem_desc_sw128(th + 32 * k), db, idesc, k ? 1u : 0u);
                    tc_mma(acc, smem_desc_sw128(tm + 32 * k), db, idesc, 1u);
                    if constexpr (kTcTerms == 3) tc_mma(acc, smem_desc_sw128(tl + 32 * k), db, idesc, 1u);
                }
            } else {
                const uint32_t bh = sa + kTcM * 128, bm = bh + N * 128, bl = bm + N * 128;
#pragma unroll
                for (int k = 0; k < kTcK / 16; ++k) {  // 16 BF16 = 32 bytes per MMA K step
                    const uint64_t da = smem_desc_sw128(sa + 32 * k);
                    tc_mma(acc, da, smem_desc_sw128(bh + 32 * k), idesc, k ? 1u : 0u);
                    tc_mma(acc, da, smem_desc_sw128(bm + 32 * k), idesc, 1u);
                    if constexpr (kTcTerms == 3) tc_mma(acc, da, smem_desc_sw128(bl + 32 * k), idesc, 1u);
                }
            }
            tc_commit(&empty_bar[s]);   // the stage is free once these MMAs have read it
            tc_commit(&acc_full[a]);    // and the block's partial is ready
            if (++s == static_cast<uint32_t>(stages)) {
                s = 0;
                phase ^= 1u;
            }
        }
    } else if (warp >= 2) {
        constexpr int C0 = tc_fold_split<N>();
        const TcEpilogue e{p, tmem, static_cast<uint32_t>(warp), static_cast<uint32_t>(lane), kblocks, acc_full,
                           acc_empty, &abort_flag, base, row0, tok0};
        if constexpr (C0 < N) {
            if ((warp - 2) / 4 == 0) tc_fold_store<N, TOKM, 0, C0, kTcAcc, kStride>(e);
            else tc_fold_store<N, TOKM, C0, N - C0, kTcAcc, kStride>(e);
        } else {
            tc_fold_store<N, TOKM, 0, N, kTcAcc, kStride>(e);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols) : "memory");
    }
}

// y[t][r] = sum over z (in order) of part[z][t][r].
__global__ void splitk_sum_kernel(const float *part, uint32_t splits, uint32_t T, uint32_t R, float *y, uint64_t ys) {
    pdl_launch_dependents();
    pdl_wait();
    const uint64_t total = static_cast<uint64_t>(T) * R, plane = total;
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        float s = part[i];
        for (uint32_t z = 1; z < splits; ++z) s = __fadd_rn(s, part[z * plane + i]);
        const uint64_t t = i / R, r = i - t * R;
        y[t * ys + r] = s;
    }
}

// FP32 rows -> BF16 terms hi = bf16(x), mid = bf16(x - hi), lo = bf16(x - hi - mid)
// (round to nearest even), row stride xs, outputs [T][K] contiguous.
__global__ void split_hilo_kernel(const float *x, uint64_t xs, uint32_t T, uint32_t K, uint16_t *hi, uint16_t *mid,
                                  uint16_t *lo) {
    pdl_launch_dependents();
    pdl_wait();
    const uint64_t total = static_cast<uint64_t>(T) * K;
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint64_t t = i / K, k = i - t * K;
        const float v = x[t * xs + k];
        const uint16_t h = plamo_bf16_round(v);
        const float r1 = __fsub_rn(v, __uint_as_float(static_cast<uint32_t>(h) << 16));
        const uint16_t md = plamo_bf16_round(r1);
        const float r2 = __fsub_rn(r1, __uint_as_float(static_cast<uint32_t>(md) << 16));
        hi[i] = h;
        mid[i] = md;
        lo[i] = plamo_bf16_round(r2);
    }
}

}  // namespace plamo
