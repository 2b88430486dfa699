// Q/K head norm + RoPE, GQA attention over the KV ring, KV ring stores.
//
// KV layout in HBM (per layer): a ring of `ring` slots of normalised,
// UNROTATED FP32 keys and values, exactly the rows the reference keeps in
// struct cache (reference src/cache.s), stored in pages of kKvPageRows slots
// taken from a page pool the backend shares between requests: the layer's
// page table maps slot s to page pages[s / kKvPageRows], whose first half
// holds the keys [kKvPageRows][kh*dim] and second half the values. Logical
// row p (0-based count of rows appended in the request) lives in slot
// p % ring. A sliding layer keeps the last `capacity` rows; instead of the
// reference's shift-and-rerotate of the whole window on every eviction
// (src/cache.s:15-63, src/cache_rope.s:12-37, kernels.metal:763-787), the
// attention kernel rotates each key on the fly at its LOCAL position
// (row - window start) from an exact host-built cos/sin table, which yields
// the same rotated keys as the reference's rotation cache with no O(window)
// copy per token.
//
// The rows of the tokens being processed (1 for decode, T for prefill, the
// candidates of a verification) are read from the QKV projection buffer, so a
// prefill longer than a sliding window never overwrites rows that an earlier
// query of the same batch still needs; they are stored into the ring after
// attention.
#pragma once
#include <cooperative_groups.h>

#include "common.cuh"
#include "rows.cuh"

namespace plamo {

constexpr uint64_t kKvPageRows = 64;

struct AttnLayer {
    float *const *pages;           // page table: [ring / kKvPageRows] page bases ([2][kKvPageRows][kvw] floats)
    uint64_t kvw;                  // floats per K (or V) row: kh*dim
    const uint64_t *appended;      // device counter: rows committed before this call
    uint64_t ring, capacity;
    int sliding;
    const float *table;  // [positions][dim]: cos[dim/2] | sin[dim/2], scale applied
    uint64_t positions;
    const uint16_t *qn, *kn;
};

struct AttnShape {
    uint64_t tokens, qh, kh, dim;
    uint64_t qkv_stride;  // floats between token rows of the QKV buffer
};

// The key and value rows of logical row `row` (slot row % ring).
__device__ __forceinline__ float *kv_key(const AttnLayer &L, uint64_t row) {
    const uint64_t s = row % L.ring;
    return L.pages[s / kKvPageRows] + (s % kKvPageRows) * L.kvw;
}
__device__ __forceinline__ float *kv_value(const AttnLayer &L, uint64_t row) {
    const uint64_t s = row % L.ring;
    return L.pages[s / kKvPageRows] + (kKvPageRows + s % kKvPageRows) * L.kvw;
}

__device__ __forceinline__ uint64_t window_start(const AttnLayer &L, uint64_t P, uint64_t t) {
    if (!L.sliding) return 0;
    const uint64_t end = P + t + 1;
    return end > L.capacity ? end - L.capacity : 0;
}

// Per (head, token): RMSNorm(+1) of Q and K heads in place; Q heads are also
// rotated at their local position into q_out [tokens][qh][dim]. V untouched.
// (reference src/qkv.s:36-70 norm, src/rope.s rotation, src/mixer.s:60-65).
__global__ void qk_prep_kernel(float *qkv, float *q_out, AttnLayer L, AttnShape S) {
    __shared__ float red[32];
    __shared__ float xn[512];
    pdl_wait();
    const uint64_t head = blockIdx.x, t = blockIdx.y, D = S.dim, half = D / 2;
    float *x = qkv + t * S.qkv_stride + head * D;
    const uint16_t *w = head < S.qh ? L.qn : L.kn;
    float s = 0.0f;
    for (uint64_t i = threadIdx.x; i < D; i += blockDim.x) s += x[i] * x[i];
    const float inv = rms_inverse(block_sum(s, red), D);
    for (uint64_t i = threadIdx.x; i < D; i += blockDim.x) xn[i] = rms_apply(x[i], inv, w[i], 1.0f);
    __syncthreads();
    if (head < S.qh) {
        const uint64_t P = *L.appended;
        const uint64_t pos = P + t - window_start(L, P, t);
        const float *c = L.table + pos * D, *sn = c + half;
        float *o = q_out + (t * S.qh + head) * D;
        for (uint64_t i = threadIdx.x; i < half; i += blockDim.x) {
            const float a = xn[i], b = xn[i + half];
            o[i] = __fsub_rn(__fmul_rn(a, c[i]), __fmul_rn(b, sn[i]));
            o[i + half] = __fadd_rn(__fmul_rn(b, c[i]), __fmul_rn(a, sn[i]));
        }
    } else {
        for (uint64_t i = threadIdx.x; i < D; i += blockDim.x) x[i] = xn[i];
    }
    pdl_launch_dependents();
}

// Head dim 128: one warp per head, eight heads per CTA, with the decode
// attention kernel's lane layout and reduction order, so prompt and decode
// normalise (and rotate) Q and K to the same bits: a Q head's lanes l < 16
// hold dims 4l..4l+3 and 64+4l..64+4l+3; a K head's 32 lanes hold 4l..4l+3.
__global__ void __launch_bounds__(256) qk_prep128_kernel(float *qkv, float *q_out, AttnLayer L, AttnShape S) {
    constexpr uint32_t D = 128, H = 64;
    pdl_wait();
    const uint32_t lane = threadIdx.x & 31;
    const uint64_t head = static_cast<uint64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5), t = blockIdx.y;
    if (head < S.qh) {
        const float *x = qkv + t * S.qkv_stride + head * D;
        const uint64_t P = *L.appended;
        const float *table = L.table + (P + t - window_start(L, P, t)) * D;
        float4 a = make_float4(0, 0, 0, 0), b = a, c = a, sn = a;
        uint2 wa = make_uint2(0, 0), wb = wa;
        if (lane < 16) {
            a = ld4(x + 4 * lane);
            b = ld4(x + H + 4 * lane);
            wa = *reinterpret_cast<const uint2 *>(L.qn + 4 * lane);
            wb = *reinterpret_cast<const uint2 *>(L.qn + H + 4 * lane);
            c = ld4(table + 4 * lane);
            sn = ld4(table + H + 4 * lane);
        }
        const float inv = rms_inverse(warp_sum(sq4(a) + sq4(b)), D);
        if (lane < 16) {
            const float4 qa = apply4(a, inv, norm4(wa, 1.0f)), qb = apply4(b, inv, norm4(wb, 1.0f));
            float4 lo4, hi4;
            lo4.x = __fsub_rn(__fmul_rn(qa.x, c.x), __fmul_rn(qb.x, sn.x));
            lo4.y = __fsub_rn(__fmul_rn(qa.y, c.y), __fmul_rn(qb.y, sn.y));
            lo4.z = __fsub_rn(__fmul_rn(qa.z, c.z), __fmul_rn(qb.z, sn.z));
            lo4.w = __fsub_rn(__fmul_rn(qa.w, c.w), __fmul_rn(qb.w, sn.w));
            hi4.x = __fadd_rn(__fmul_rn(qb.x, c.x), __fmul_rn(qa.x, sn.x));
            hi4.y = __fadd_rn(__fmul_rn(qb.y, c.y), __fmul_rn(qa.y, sn.y));
            hi4.z = __fadd_rn(__fmul_rn(qb.z, c.z), __fmul_rn(qa.z, sn.z));
            hi4.w = __fadd_rn(__fmul_rn(qb.w, c.w), __fmul_rn(qa.w, sn.w));
            float *o = q_out + (t * S.qh + head) * D;
            *reinterpret_cast<float4 *>(o + 4 * lane) = lo4;
            *reinterpret_cast<float4 *>(o + H + 4 * lane) = hi4;
        }
    } else if (head < S.qh + S.kh) {
        float *x = qkv + t * S.qkv_stride + head * D;
        const float4 xk = ld4(x + 4 * lane);
        const uint2 wk = *reinterpret_cast<const uint2 *>(L.kn + 4 * lane);
        const float inv = rms_inverse(warp_sum(sq4(xk)), D);
        *reinterpret_cast<float4 *>(x + 4 * lane) = apply4(xk, inv, norm4(wk, 1.0f));
    }
    pdl_launch_dependents();
}

constexpr int kAttnThreads = 128;
constexpr int kAttnTile = 32;

struct AttnParams {
    AttnLayer L;
    AttnShape S;
    const float *q;    // [tokens][qh][dim], rotated
    const float *qkv;  // new rows: K at qh*dim, V at (qh+kh)*dim of each token row
    float *out;        // [tokens][qh][dim]
    float *part;       // [tokens][qh][splits][dim + 2] partial (acc, m, l)
    uint32_t *tickets; // [tokens][kh] arrival counters (zero between launches)
    uint32_t splits;
    uint32_t t0;       // first query token of this launch (blockIdx.y counts from it)
    // When set, the output's BF16 terms for the next projection (three planes
    // split_plane apart, indexed as out).
    uint16_t *split = nullptr;
    uint64_t split_plane = 0;
};

// One CTA per (kv head, query token, key split). Keys of the split are
// staged in tiles of 32 rows, rotated at their local position, scored against
// the G = qh/kh query heads of the group, and folded into an online softmax
// whose exponentials are the reference's exp polynomial. The last CTA of a
// (token, kv head) merges the split partials in split order.
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(AttnParams p) {
    extern __shared__ __align__(16) float sm[];
    const uint32_t D = static_cast<uint32_t>(p.S.dim), half = D / 2;
    const uint32_t QH = static_cast<uint32_t>(p.S.qh), KH = static_cast<uint32_t>(p.S.kh), G = QH / KH;
    const uint64_t kh = blockIdx.x, t = blockIdx.y + p.t0, split = blockIdx.z;
    const uint32_t KS = D + 1;          // padded key row: conflict-free column reads
    float *qs = sm;                     // [G][D]
    float *kt = qs + G * D;             // [tile][D + 1]
    float *vt = kt + kAttnTile * KS;    // [tile][D]
    float *sc = vt + kAttnTile * D;     // [G][tile]
    float *acc = sc + G * kAttnTile;    // [G][D]
    float *mrow = acc + G * D;          // [G]
    float *lrow = mrow + G;             // [G]
    float *corr = lrow + G;             // [G]
    __shared__ uint32_t is_last;

    pdl_wait();
    const uint64_t P = *p.L.appended;
    const uint64_t lo = window_start(p.L, P, t), hi = P + t + 1;  // keys [lo, hi)
    const uint64_t n = hi - lo;
    const uint64_t k0 = lo + n * split / p.splits, k1 = lo + n * (split + 1) / p.splits;
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(D)));

    for (uint64_t i = threadIdx.x; i < G * D; i += blockDim.x) {
        const uint64_t g = i / D, d = i % D;
        qs[i] = p.q[(t * QH + kh * G + g) * D + d];
        acc[i] = 0.0f;
    }
    for (uint64_t g = threadIdx.x; g < G; g += blockDim.x) {
        mrow[g] = -__int_as_float(0x7f800000);
        lrow[g] = 0.0f;
    }
    __syncthreads();

    for (uint64_t base = k0; base < k1; base += kAttnTile) {
        const uint64_t rows = k1 - base < kAttnTile ? k1 - base : kAttnTile;
        // Stage rotated keys and values of the tile.
        for (uint32_t i = threadIdx.x; i < rows * half; i += blockDim.x) {
            const uint32_t r = i / static_cast<uint32_t>(half), d = i - r * static_cast<uint32_t>(half);
            const uint64_t key = base + r;
            const float *ksrc, *vsrc;
            if (key < P) {
                ksrc = kv_key(p.L, key) + kh * D;
                vsrc = kv_value(p.L, key) + kh * D;
            } else {
                const float *row = p.qkv + (key - P) * p.S.qkv_stride;
                ksrc = row + QH * D + kh * D;
                vsrc = row + (QH + KH) * D + kh * D;
            }
            const float *c = p.L.table + (key - lo) * D, *s = c + half;
            const float a = ksrc[d], b = ksrc[d + half];
            kt[r * KS + d] = __fsub_rn(__fmul_rn(a, c[d]), __fmul_rn(b, s[d]));
            kt[r * KS + d + half] = __fadd_rn(__fmul_rn(b, c[d]), __fmul_rn(a, s[d]));
            vt[r * D + d] = vsrc[d];
            vt[r * D + d + half] = vsrc[d + half];
        }
        __syncthreads();
        // Scores: sequential FMA over dim per (head, key), times 1/sqrt(dim).
        for (uint32_t i = threadIdx.x; i < G * rows; i += blockDim.x) {
            const uint32_t g = i / static_cast<uint32_t>(rows), r = i - g * static_cast<uint32_t>(rows);
            const float *qv = qs + g * D, *kv = kt + r * KS;
            float a = 0.0f;
            for (uint32_t d = 0; d < D; ++d) a = fmaf(qv[d], kv[d], a);
            sc[g * kAttnTile + r] = __fmul_rn(a, scale);
        }
        __syncthreads();
        // Online softmax bookkeeping, one thread per head.
        for (uint64_t g = threadIdx.x; g < G; g += blockDim.x) {
            float m = mrow[g];
            for (uint64_t r = 0; r < rows; ++r) m = fmaxf(m, sc[g * kAttnTile + r]);
            const float c = plamo_exp(__fsub_rn(mrow[g], m));
            float l = __fmul_rn(lrow[g], c);
            for (uint64_t r = 0; r < rows; ++r) {
                const float e = plamo_exp(__fsub_rn(sc[g * kAttnTile + r], m));
                sc[g * kAttnTile + r] = e;
                l = __fadd_rn(l, e);
            }
            mrow[g] = m;
            lrow[g] = l;
            corr[g] = c;
        }
        __syncthreads();
        // Weighted values: sequential FMA over the tile's keys.
        for (uint32_t i = threadIdx.x; i < G * D; i += blockDim.x) {
            const uint32_t g = i / static_cast<uint32_t>(D), d = i - g * static_cast<uint32_t>(D);
            float a = __fmul_rn(acc[i], corr[g]);
            for (uint32_t r = 0; r < rows; ++r) a = fmaf(sc[g * kAttnTile + r], vt[r * D + d], a);
            acc[i] = a;
        }
        __syncthreads();
    }

    if (p.splits == 1) {
        for (uint64_t i = threadIdx.x; i < G * D; i += blockDim.x) {
            const uint64_t g = i / D, d = i % D;
            const float o = __fdiv_rn(acc[i], lrow[g]);
            const uint64_t at = (t * QH + kh * G + g) * D + d;
            p.out[at] = o;
            if (p.split) split3(o, p.split + at, p.split + p.split_plane + at, p.split + 2 * p.split_plane + at);
        }
        pdl_launch_dependents();
        return;
    }
    const uint64_t pstride = D + 2;
    for (uint64_t i = threadIdx.x; i < G * D; i += blockDim.x) {
        const uint64_t g = i / D, d = i % D;
        p.part[((t * QH + kh * G + g) * p.splits + split) * pstride + d] = acc[i];
    }
    for (uint64_t g = threadIdx.x; g < G; g += blockDim.x) {
        float *slot = p.part + ((t * QH + kh * G + g) * p.splits + split) * pstride + D;
        slot[0] = mrow[g];
        slot[1] = lrow[g];
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const uint32_t ticket = atomicAdd(&p.tickets[t * KH + kh], 1u);
        is_last = ticket == p.splits - 1;
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    // Merge in split order: M = max m_s, L = sum l_s e^(m_s - M),
    // out = sum acc_s e^(m_s - M) / L.
    for (uint64_t i = threadIdx.x; i < G * D; i += blockDim.x) {
        const uint64_t g = i / D, d = i % D;
        const float *base = p.part + (t * QH + kh * G + g) * p.splits * pstride;
        float M = -__int_as_float(0x7f800000);
        for (uint32_t s = 0; s < p.splits; ++s) M = fmaxf(M, base[s * pstride + D]);
        float Ls = 0.0f, A = 0.0f;
        for (uint32_t s = 0; s < p.splits; ++s) {
            const float e = plamo_exp(__fsub_rn(base[s * pstride + D], M));
            Ls = fmaf(base[s * pstride + D + 1], e, Ls);
            A = fmaf(base[s * pstride + d], e, A);
        }
        const float o = __fdiv_rn(A, Ls);
        const uint64_t at = (t * QH + kh * G + g) * D + d;
        p.out[at] = o;
        if (p.split) split3(o, p.split + at, p.split + p.split_plane + at, p.split + 2 * p.split_plane + at);
    }
    __syncthreads();
    if (threadIdx.x == 0) p.tickets[t * KH + kh] = 0;
    pdl_launch_dependents();
}

inline size_t attention_smem_bytes(uint64_t G, uint64_t D) {
    return (G * D + kAttnTile * (D + 1) + kAttnTile * D + G * kAttnTile + G * D + 3 * G) *
           sizeof(float);
}

// ---------------------------------------------------------------------------
// Prompt attention, blocked over queries (dim 128). attention_kernel stages
// and rotates every key once per query token; here every key of the layer is
// rotated once (prompt_keys_kernel), and one CTA takes 64 query rows (64/G
// consecutive tokens x the G heads of one kv head) so that every staged key
// tile serves all of them, from registers:
//   staging - rotated keys and values of the next tile are copied with
//             cp.async (16-byte pieces) into the other half of a double
//             buffer while the current tile is computed;
//   scores  - each thread 4 rows x 2 keys, Q transposed in shared memory
//             (one 128-bit load per 4 rows and dim), keys read as 128-bit
//             words of four dims (rows padded to 132 floats: the 8 threads of
//             a quarter warp cover all 32 banks);
//   softmax - row max by shuffles over the 16 threads of a row group, the
//             reference exp per element, row sums sequential in key order;
//   values  - each thread 8 rows x 4 dims, acc *= correction then sequential
//             FMA over the tile's keys.
// The arithmetic is attention_kernel's with one split, operation for
// operation: keys rotated with the same products and roundings, 32-key tiles
// from the window start, sequential FMA dots over dim (dim 0 first) times
// 1/sqrt(dim), running max, l = l*c + e in key order, acc = acc*c then FMA in
// key order, out = acc / l. Keys past a row's causal end enter as
// exp(-inf) = 0, which leaves l, the max and acc unchanged, so every output
// is bit-identical to attention_kernel's and independent of how the prompt is
// batched. All queries of one launch must share the window start 0 (full
// layers, or sliding layers whose window is not yet full); the host sends the
// other queries of a sliding layer to attention_kernel.
constexpr int kPaThreads = 256;
constexpr int kPaRows = 64;             // query rows (token x head) per CTA, at most
constexpr int kPaTile = kAttnTile;      // keys per tile
constexpr int kPaD = 128;
constexpr int kPaKS = kPaD + 4;         // padded key row (16-byte multiple, conflict-free 128-bit reads)

struct PromptAttnParams {
    AttnLayer L;
    const float *q;     // [tokens][qh][128], rotated
    const float *qkv;   // new rows: K at qh*128, V at (qh+kh)*128 of each token row
    const float *rotk;  // [keys][kh*128] rotated keys of rows [0, P + tokens) (prompt_keys_kernel)
    float *out;         // [tokens][qh][128]
    uint32_t qh, kh, qkv_stride;
    uint32_t tokens;     // queries [0, tokens) of this call
    uint32_t per_block;  // query tokens per CTA: rows per CTA / G
    uint16_t *split;     // the output's BF16 terms for the next projection (planes split_plane apart), or null
    uint64_t split_plane;
};

// Keys [0, keys) of a layer whose window starts at row 0, each rotated at its
// own row (cached rows from the ring, new rows from the normalised K of the
// projection), with attention_kernel's in-tile products and roundings.
__global__ void prompt_keys_kernel(AttnLayer L, const float *qkv, uint32_t qkv_stride, uint32_t qh, uint32_t kh,
                                   float *rotk, uint32_t keys) {
    constexpr uint32_t D = kPaD, half = kPaD / 2;
    pdl_wait();
    const uint64_t P = *L.appended;
    const uint64_t kvw = static_cast<uint64_t>(kh) * D;
    const uint64_t total = static_cast<uint64_t>(keys) * kh * half;
    for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint32_t d = static_cast<uint32_t>(i % half);
        const uint64_t rest = i / half, key = rest / kh, h = rest % kh;
        const float *src = key < P ? kv_key(L, key) + h * D
                                   : qkv + (key - P) * qkv_stride + static_cast<uint64_t>(qh) * D + h * D;
        const float *c = L.table + key * D, *s = c + half;
        const float a = src[d], b = src[d + half];
        float *o = rotk + key * kvw + h * D;
        o[d] = __fsub_rn(__fmul_rn(a, c[d]), __fmul_rn(b, s[d]));
        o[d + half] = __fadd_rn(__fmul_rn(b, c[d]), __fmul_rn(a, s[d]));
    }
    pdl_launch_dependents();
}

// Shared memory of a CTA of ROWS query rows (BUFS key/value tile buffers).
template <int ROWS, int BUFS = 2>
constexpr size_t prompt_attention_smem_bytes() {
    return (kPaD * (ROWS + 4) + BUFS * kPaTile * kPaKS + BUFS * kPaTile * kPaD + kPaTile * (ROWS + 4) + 2 * ROWS) *
           sizeof(float);
}

// ROWS query rows per CTA (64, or 32 for short prompts: twice the CTAs,
// half the work per key tile, so the longest blocks finish sooner). Every
// row's operations are the same for either ROWS.
template <int ROWS, int BUFS = 2>
__global__ void __launch_bounds__(kPaThreads) prompt_attention_kernel(PromptAttnParams p) {
    static_assert(ROWS == 64 || ROWS == 32, "64 or 32 query rows per CTA");
    static_assert(BUFS == 1 || BUFS == 2, "one or two tile buffers");
    constexpr int QS = ROWS + 4;       // transposed Q / P row stride (16-byte multiple)
    constexpr int RT = ROWS / 16;      // score phase: rows per thread (16 row groups)
    constexpr int RW = ROWS / 8;       // value phase: rows per warp (8 warps)
    extern __shared__ __align__(16) float sm[];
    float *qT = sm;                        // [128][QS]  Q rows, transposed
    float *kt = qT + kPaD * QS;               // [BUFS][tile][kPaKS] rotated keys
    float *vt = kt + BUFS * kPaTile * kPaKS;  // [BUFS][tile][128]   values
    float *pT = vt + BUFS * kPaTile * kPaD;   // [tile][QS] exp(score - max), transposed
    float *corr = pT + kPaTile * QS;       // [ROWS] per-row correction of the tile
    float *lsum = corr + ROWS;             // [ROWS] final row sums
    constexpr uint32_t D = kPaD;
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t G = p.qh / p.kh, BQ = p.per_block;
    const uint32_t kh = blockIdx.y;
    const uint32_t t0 = (gridDim.x - 1 - blockIdx.x) * BQ;  // latest (longest) blocks start first
    const uint32_t tq = min(BQ, p.tokens - t0), vrows = tq * G;
    const uint64_t kvw = static_cast<uint64_t>(p.kh) * D;
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(D)));
    const float ninf = -__int_as_float(0x7f800000);

    pdl_wait();
    const uint32_t P = static_cast<uint32_t>(*p.L.appended);
    const uint32_t hi_max = P + t0 + tq;  // keys [0, hi_max)

    // Asynchronous copy of the rotated keys and the values of one tile.
    auto stage = [&](uint32_t base, uint32_t buf) {
        const uint32_t trow = min(static_cast<uint32_t>(kPaTile), hi_max - base);
        float *ktb = kt + buf * (kPaTile * kPaKS), *vtb = vt + buf * (kPaTile * kPaD);
        for (uint32_t i = tid; i < trow * (D / 4); i += kPaThreads) {
            const uint32_t r = i / (D / 4), c = (i - r * (D / 4)) * 4, key = base + r;
            cp_async16(ktb + r * kPaKS + c, p.rotk + key * kvw + kh * D + c);
            const float *vsrc = key < P ? kv_value(p.L, key) + kh * D
                                        : p.qkv + static_cast<size_t>(key - P) * p.qkv_stride + (p.qh + p.kh) * D +
                                              kh * D;
            cp_async16(vtb + r * D + c, vsrc + c);
        }
        cp_async_commit();
    };
    stage(0, 0);

    for (uint32_t i = tid; i < ROWS * D; i += kPaThreads) {
        const uint32_t r = i / D, d = i - r * D;
        float v = 0.0f;
        if (r < vrows) {
            const uint32_t qi = r / G, g = r - qi * G;
            v = p.q[(static_cast<size_t>(t0 + qi) * p.qh + kh * G + g) * D + d];
        }
        qT[d * QS + r] = v;
    }

    // Score-phase roles: rows ty*RT .. ty*RT+RT-1, keys tx and tx+16.
    const uint32_t ty = tid >> 4, tx = tid & 15;
    uint32_t hi[RT];
#pragma unroll
    for (int i = 0; i < RT; ++i) {
        const uint32_t r = ty * RT + i;
        hi[i] = r < vrows ? P + t0 + r / G + 1 : 0;
    }
    float mrow[RT];
#pragma unroll
    for (int i = 0; i < RT; ++i) mrow[i] = ninf;
    // Value-phase roles: rows warp*RW .. warp*RW+RW-1, dims lane*4 .. lane*4+3.
    float acc[RW][4];
#pragma unroll
    for (int i = 0; i < RW; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;
    float l = 0.0f;  // row `tid` (tid < ROWS)

    uint32_t buf = 0;
    for (uint32_t base = 0; base < hi_max; base += kPaTile, buf ^= (BUFS - 1)) {
        const uint32_t trow = min(static_cast<uint32_t>(kPaTile), hi_max - base);
        if (BUFS == 2 && base + kPaTile < hi_max) {
            stage(base + kPaTile, buf ^ 1u);  // that half was released by the last iteration's barrier
            cp_async_wait_one();
        } else {
            if (BUFS == 1 && base > 0) stage(base, 0);  // the single buffer was released by the last barrier
            cp_async_wait_all();
        }
        __syncthreads();
        const float *ktb = kt + buf * (kPaTile * kPaKS), *vtb = vt + buf * (kPaTile * kPaD);

        float s[RT][2];
#pragma unroll
        for (int i = 0; i < RT; ++i) s[i][0] = s[i][1] = 0.0f;
        const float *k0 = ktb + tx * kPaKS, *k1 = ktb + (tx + 16) * kPaKS;
#pragma unroll 2
        for (uint32_t d = 0; d < D; d += 4) {
            const float4 a4 = *reinterpret_cast<const float4 *>(k0 + d);
            const float4 b4 = *reinterpret_cast<const float4 *>(k1 + d);
            const float ka[4] = {a4.x, a4.y, a4.z, a4.w}, kb[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                float q[RT];
                if constexpr (RT == 4) {
                    const float4 q4 = *reinterpret_cast<const float4 *>(qT + (d + e) * QS + ty * 4);
                    q[0] = q4.x;
                    q[1] = q4.y;
                    q[2] = q4.z;
                    q[3] = q4.w;
                } else {
                    const float2 q2 = *reinterpret_cast<const float2 *>(qT + (d + e) * QS + ty * 2);
                    q[0] = q2.x;
                    q[1] = q2.y;
                }
#pragma unroll
                for (int i = 0; i < RT; ++i) {
                    s[i][0] = fmaf(q[i], ka[e], s[i][0]);
                    s[i][1] = fmaf(q[i], kb[e], s[i][1]);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < RT; ++i) {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const uint32_t key = base + tx + 16 * j;
                s[i][j] = key < hi[i] ? __fmul_rn(s[i][j], scale) : ninf;
            }
            float m = fmaxf(s[i][0], s[i][1]);
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            m = fmaxf(mrow[i], m);
            const float c = plamo_exp(__fsub_rn(mrow[i], m));
            mrow[i] = m;
            pT[tx * QS + ty * RT + i] = plamo_exp(__fsub_rn(s[i][0], m));
            pT[(tx + 16) * QS + ty * RT + i] = plamo_exp(__fsub_rn(s[i][1], m));
            if (tx == 0) corr[ty * RT + i] = c;
        }
        __syncthreads();

        if (tid < ROWS) {
            l = __fmul_rn(l, corr[tid]);
            for (uint32_t r = 0; r < trow; ++r) l = __fadd_rn(l, pT[r * QS + tid]);
        }
#pragma unroll
        for (int i = 0; i < RW; ++i) {
            const float c = corr[warp * RW + i];
            acc[i][0] = __fmul_rn(acc[i][0], c);
            acc[i][1] = __fmul_rn(acc[i][1], c);
            acc[i][2] = __fmul_rn(acc[i][2], c);
            acc[i][3] = __fmul_rn(acc[i][3], c);
        }
        for (uint32_t r = 0; r < trow; ++r) {
            const float4 v = *reinterpret_cast<const float4 *>(vtb + r * D + lane * 4);
            float pr[RW];
#pragma unroll
            for (int h = 0; h < RW; h += 4) {
                const float4 p4 = *reinterpret_cast<const float4 *>(pT + r * QS + warp * RW + h);
                pr[h] = p4.x;
                pr[h + 1] = p4.y;
                pr[h + 2] = p4.z;
                pr[h + 3] = p4.w;
            }
#pragma unroll
            for (int i = 0; i < RW; ++i) {
                acc[i][0] = fmaf(pr[i], v.x, acc[i][0]);
                acc[i][1] = fmaf(pr[i], v.y, acc[i][1]);
                acc[i][2] = fmaf(pr[i], v.z, acc[i][2]);
                acc[i][3] = fmaf(pr[i], v.w, acc[i][3]);
            }
        }
        __syncthreads();
    }

    if (tid < ROWS) lsum[tid] = l;
    __syncthreads();
#pragma unroll
    for (int i = 0; i < RW; ++i) {
        const uint32_t r = warp * RW + i;
        if (r >= vrows) continue;
        const uint32_t qi = r / G, g = r - qi * G;
        const float inv = lsum[r];
        float4 o = make_float4(__fdiv_rn(acc[i][0], inv), __fdiv_rn(acc[i][1], inv), __fdiv_rn(acc[i][2], inv),
                               __fdiv_rn(acc[i][3], inv));
        const uint64_t at = (static_cast<uint64_t>(t0 + qi) * p.qh + kh * G + g) * D + lane * 4;
        *reinterpret_cast<float4 *>(p.out + at) = o;
        if (p.split) {
            RowFuse f{};
            f.split = p.split;
            fuse_split4(f, p.split_plane, at, o);
        }
    }
    pdl_launch_dependents();
}

// ---------------------------------------------------------------------------
// Decode attention, fused: one launch per layer does the Q/K head RMSNorm and
// RoPE of the new token, attention over the window with keys rotated on the
// fly, and the store of the new K/V row into the ring.
//
// Grid (kv head, 8 key splits); the 8 splits of a kv head form one thread
// block cluster. Every CTA normalises and rotates the G query heads of its
// group itself (a few KB from L2); the CTA whose split ends at the new row
// also normalises its key and writes K and V to ring slot P % ring (no CTA of
// this launch reads that slot: it holds a row outside every window). Scores
// are sequential FMA dots over dim, as the reference computes them; softmax
// is online per tile with the reference's exp. The split partials stay in
// shared memory and cluster rank 0 merges them through distributed shared
// memory (no global round trip, no atomics).
constexpr int kDecThreads = 256;
constexpr int kDecTile = 64;
constexpr int kDecSplits = 8;
// Head dim 128, one request: 16 key splits per KV head (a non-portable
// cluster of 16), so a context of up to 1024 rows is one tile per CTA.
// Several requests in one launch already fill the GPU with clusters, and
// measured faster with 8 splits each (4.80 against 4.95 ms per 8-request
// 8B step).
constexpr int kDec128Splits = 16;
constexpr uint32_t kDecPageCache = 64;  // page bases held in shared memory (rows 0..4095 of a ring)
constexpr int kDec128BatchSplits = 8;

struct DecodeAttnParams {
    AttnLayer L;
    uint32_t qh, kh, dim;
    float *qkv;  // [qh + 2 kh][dim] projection of the token (read only)
    float *out;  // [qh][dim]
    unsigned long long *trace = nullptr;  // launch timeline record (trace_stamp), or null
};

// Key tile row stride: D + 4 keeps 16-byte alignment and spreads the rows of
// eight lanes over all 32 banks for 128-bit reads (D = 128), D + 1 for any D.
__host__ __device__ inline uint32_t decode_key_stride(uint32_t D) { return D % 8 == 0 ? D + 4 : D + 1; }

inline size_t decode_attention_smem(uint32_t G, uint32_t D) {
    return sizeof(float) * (static_cast<size_t>(G) * D                     // qs
                            + kDecTile * decode_key_stride(D)              // kt
                            + kDecTile * D                                 // vt
                            + G * kDecTile                                 // sc
                            + G * D                                        // acc
                            + 2 * D                                        // knew, vnew
                            + 3 * G);                                      // m, l, corr
}

// Head dim 128: every load of a tile is an asynchronous 16-byte copy issued
// before any compute (raw keys into the padded key tile, values, and the
// tile's cos/sin rows, which are consecutive table rows), the Q/K head norms
// run while they are in flight, and keys are then rotated in place.
constexpr uint32_t kD128Stride = 132;
inline size_t decode_attention128_smem(uint32_t G) {
    return sizeof(float) * (static_cast<size_t>(G) * 128  // qs
                            + kDecTile * kD128Stride      // kt (raw, then rotated in place)
                            + kDecTile * 128              // tab (cos | sin rows)
                            + kDecTile * 128              // vt
                            + G * kDecTile                // sc
                            + G * 128                     // acc
                            + 2 * 128                     // knew, vnew
                            + 3 * G);
}

template <int S>
__device__ __forceinline__ void decode_attention128_body(const DecodeAttnParams &p) {
    static_assert(S >= 2 && 32 % S == 0, "a head's splits share one warp in the merge");
    constexpr uint32_t D = 128, H = 64, KS = kD128Stride;
    extern __shared__ __align__(16) float sm[];
    const uint32_t G = p.qh / p.kh;
    const uint32_t kh = blockIdx.x, split = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = kDecThreads / 32;
    float *qs = sm;
    float *kt = qs + G * D;
    float *tab = kt + kDecTile * KS;
    float *vt = tab + kDecTile * D;
    float *sc = vt + kDecTile * D;
    float *acc = sc + G * kDecTile;
    float *knew = acc + G * D;
    float *vnew = knew + D;
    float *mrow = vnew + D;
    float *lrow = mrow + G;
    float *corr = lrow + G;
    cooperative_groups::cluster_group cluster = cooperative_groups::this_cluster();
    const uint64_t t_entry = p.trace ? global_ns() : 0;

    pdl_launch_dependents();  // the next projection may start streaming its weights
    // The committed rows and their counter were final before this step began
    // (only the new row comes from the projection still in flight), and so
    // were the page table's entries, so the first tile of old rows is
    // requested before waiting for that projection. The first pages' bases
    // are read into shared memory alongside the counter, keeping the page
    // lookups off the chain of dependent global loads.
    __shared__ float *page_base[kDecPageCache];
    const uint64_t npages = (p.L.ring + kKvPageRows - 1) / kKvPageRows;
    if (threadIdx.x < kDecPageCache && threadIdx.x < npages)
        page_base[threadIdx.x] =
            reinterpret_cast<float *>(load_u64_keep(p.L.pages + threadIdx.x, evict_last_policy()));
    const uint64_t P = *p.L.appended;
    const uint64_t lo = window_start(p.L, P, 0);
    const uint32_t n = static_cast<uint32_t>(P + 1 - lo);
    const uint64_t k0 = lo + static_cast<uint64_t>(n) * split / S;
    const uint64_t k1 = lo + static_cast<uint64_t>(n) * (split + 1) / S;
    __syncthreads();
    auto page_of = [&](uint64_t row, uint64_t half) -> float * {
        const uint64_t slot = row % p.L.ring, pi = slot / kKvPageRows;
        float *const base = pi < kDecPageCache ? page_base[pi] : p.L.pages[pi];
        return base + (half * kKvPageRows + slot % kKvPageRows) * p.L.kvw + kh * D;
    };
    // Where this step's new row goes (its page was mapped before the launch).
    float *const knew_dst = k1 == P + 1 ? page_of(P, 0) : nullptr;
    float *const vnew_dst = k1 == P + 1 ? page_of(P, 1) : nullptr;

    // Asynchronous staging of one tile: thread i copies columns c..c+3 and
    // c+64..c+67 (r = i / 16, c = 4 (i % 16)) of a row's key, value and
    // cos|sin entries - exactly the pairs it later rotates, so it can rotate
    // them as soon as its own copies have landed.
    auto stage = [&](uint64_t base, uint32_t rows) {
        for (uint32_t i = threadIdx.x; i < rows * 16; i += kDecThreads) {
            const uint32_t r = i >> 4, c = (i & 15) * 4;
            const uint64_t key = base + r;
            const float *trow = p.L.table + (key - lo) * D;
            cp_async16(tab + r * D + c, trow + c);
            cp_async16(tab + r * D + H + c, trow + H + c);
            if (key < P) {
                const float *krow = page_of(key, 0), *vrow = page_of(key, 1);
                cp_async16(kt + r * KS + c, krow + c);
                cp_async16(kt + r * KS + H + c, krow + H + c);
                cp_async16(vt + r * D + c, vrow + c);
                cp_async16(vt + r * D + H + c, vrow + H + c);
            }
        }
        cp_async_commit();
    };
    if (k0 < k1) stage(k0, static_cast<uint32_t>(k1 - k0 < kDecTile ? k1 - k0 : kDecTile));
    pdl_wait();
    if (p.trace && threadIdx.x == 0) {
        const uint64_t t = global_ns();
        trace_stamp(p.trace, 0, t_entry);
        trace_stamp(p.trace, 5, t_entry);
        trace_stamp(p.trace, 4, t);
        trace_stamp(p.trace, 1, t);
    }

    // Q heads of the group (one warp each): lane l < 16 owns coordinate pairs
    // 4l..4l+3 / 64+4l..64+4l+3; RMSNorm(+1), rotate at the query position.
    const float *table_q = p.L.table + static_cast<uint64_t>(n - 1) * D;
    for (uint32_t g = warp; g < G; g += warps) {
        const float *x = p.qkv + static_cast<uint64_t>(kh * G + g) * D;
        float4 a = make_float4(0, 0, 0, 0), b = a, c = a, sn = a;
        uint2 wa = make_uint2(0, 0), wb = wa;
        if (lane < 16) {
            a = ld4(x + 4 * lane);
            b = ld4(x + H + 4 * lane);
            wa = *reinterpret_cast<const uint2 *>(p.L.qn + 4 * lane);
            wb = *reinterpret_cast<const uint2 *>(p.L.qn + H + 4 * lane);
            c = ld4(table_q + 4 * lane);
            sn = ld4(table_q + H + 4 * lane);
        }
        const float inv = rms_inverse(warp_sum(sq4(a) + sq4(b)), D);
        if (lane < 16) {
            const float4 qa = apply4(a, inv, norm4(wa, 1.0f)), qb = apply4(b, inv, norm4(wb, 1.0f));
            float4 lo4, hi4;
            lo4.x = __fsub_rn(__fmul_rn(qa.x, c.x), __fmul_rn(qb.x, sn.x));
            lo4.y = __fsub_rn(__fmul_rn(qa.y, c.y), __fmul_rn(qb.y, sn.y));
            lo4.z = __fsub_rn(__fmul_rn(qa.z, c.z), __fmul_rn(qb.z, sn.z));
            lo4.w = __fsub_rn(__fmul_rn(qa.w, c.w), __fmul_rn(qb.w, sn.w));
            hi4.x = __fadd_rn(__fmul_rn(qb.x, c.x), __fmul_rn(qa.x, sn.x));
            hi4.y = __fadd_rn(__fmul_rn(qb.y, c.y), __fmul_rn(qa.y, sn.y));
            hi4.z = __fadd_rn(__fmul_rn(qb.z, c.z), __fmul_rn(qa.z, sn.z));
            hi4.w = __fadd_rn(__fmul_rn(qb.w, c.w), __fmul_rn(qa.w, sn.w));
            *reinterpret_cast<float4 *>(qs + g * D + 4 * lane) = lo4;
            *reinterpret_cast<float4 *>(qs + g * D + H + 4 * lane) = hi4;
        }
    }
    // The new row: normalised K (unrotated) and V, stored to the ring by the
    // CTA whose split contains it.
    const bool has_new = k1 == P + 1;
    // One tile (the common case): the new row goes straight into its tile row
    // (the tile's copies skip it), its key rotated here at the query's
    // position, so the tile needs no barrier before its keys are rotated.
    const bool single = k1 - k0 <= kDecTile;
    if (has_new && warp == warps - 1) {
        const float *x = p.qkv + static_cast<uint64_t>(p.qh + kh) * D;
        const float *v = p.qkv + static_cast<uint64_t>(p.qh + p.kh + kh) * D;
        const float4 xk = ld4(x + 4 * lane), xv = ld4(v + 4 * lane);
        const uint2 wk = *reinterpret_cast<const uint2 *>(p.L.kn + 4 * lane);
        const float inv = rms_inverse(warp_sum(sq4(xk)), D);
        const float4 k4 = apply4(xk, inv, norm4(wk, 1.0f));
        *reinterpret_cast<float4 *>(knew_dst + 4 * lane) = k4;
        *reinterpret_cast<float4 *>(vnew_dst + 4 * lane) = xv;
        if (single) {
            // Lane l < 16 holds dims 4l.. of the first half, lane l + 16 the
            // matching dims of the second half: the rotation pairs them.
            float4 o;
            o.x = __shfl_xor_sync(0xffffffffu, k4.x, 16);
            o.y = __shfl_xor_sync(0xffffffffu, k4.y, 16);
            o.z = __shfl_xor_sync(0xffffffffu, k4.z, 16);
            o.w = __shfl_xor_sync(0xffffffffu, k4.w, 16);
            const float4 a = lane < 16 ? k4 : o, b = lane < 16 ? o : k4;
            const float4 c = ld4(table_q + 4 * (lane & 15)), sn = ld4(table_q + H + 4 * (lane & 15));
            float4 rk;
            if (lane < 16) {
                rk.x = __fsub_rn(__fmul_rn(a.x, c.x), __fmul_rn(b.x, sn.x));
                rk.y = __fsub_rn(__fmul_rn(a.y, c.y), __fmul_rn(b.y, sn.y));
                rk.z = __fsub_rn(__fmul_rn(a.z, c.z), __fmul_rn(b.z, sn.z));
                rk.w = __fsub_rn(__fmul_rn(a.w, c.w), __fmul_rn(b.w, sn.w));
            } else {
                rk.x = __fadd_rn(__fmul_rn(b.x, c.x), __fmul_rn(a.x, sn.x));
                rk.y = __fadd_rn(__fmul_rn(b.y, c.y), __fmul_rn(a.y, sn.y));
                rk.z = __fadd_rn(__fmul_rn(b.z, c.z), __fmul_rn(a.z, sn.z));
                rk.w = __fadd_rn(__fmul_rn(b.w, c.w), __fmul_rn(a.w, sn.w));
            }
            const uint32_t rn = static_cast<uint32_t>(P - k0);
            *reinterpret_cast<float4 *>(kt + rn * KS + 4 * lane) = rk;
            *reinterpret_cast<float4 *>(vt + rn * D + 4 * lane) = xv;
        } else {
            *reinterpret_cast<float4 *>(knew + 4 * lane) = k4;
            *reinterpret_cast<float4 *>(vnew + 4 * lane) = xv;
        }
    }
    for (uint32_t i = threadIdx.x; i < G * D; i += kDecThreads) acc[i] = 0.0f;
    for (uint32_t g = threadIdx.x; g < G; g += kDecThreads) {
        mrow[g] = -__int_as_float(0x7f800000);
        lrow[g] = 0.0f;
    }

    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(D)));
    for (uint64_t base = k0; base < k1; base += kDecTile) {
        const uint32_t rows = static_cast<uint32_t>(k1 - base < kDecTile ? k1 - base : kDecTile);
        cp_async_wait_all();
        if (!single) {
            __syncthreads();
            // The new row is not in the ring yet: take it from shared memory.
            if (base + rows == P + 1) {
                const uint32_t r = rows - 1;
                for (uint32_t i = threadIdx.x; i < D; i += kDecThreads) {
                    kt[r * KS + i] = knew[i];
                    vt[r * D + i] = vnew[i];
                }
                __syncthreads();
            }
        }
        // Rotate keys in place at their local positions (tab rows): each
        // thread the pieces it staged itself (a single tile's new row is
        // already rotated).
        for (uint32_t i = threadIdx.x; i < rows * 16; i += kDecThreads) {
            const uint32_t r = i >> 4, d = (i & 15) * 4;
            if (single && base + r == P) continue;
            const float4 a = ld4(kt + r * KS + d), b = ld4(kt + r * KS + H + d);
            const float4 c = ld4(tab + r * D + d), sn = ld4(tab + r * D + H + d);
            float4 lo4, hi4;
            lo4.x = __fsub_rn(__fmul_rn(a.x, c.x), __fmul_rn(b.x, sn.x));
            lo4.y = __fsub_rn(__fmul_rn(a.y, c.y), __fmul_rn(b.y, sn.y));
            lo4.z = __fsub_rn(__fmul_rn(a.z, c.z), __fmul_rn(b.z, sn.z));
            lo4.w = __fsub_rn(__fmul_rn(a.w, c.w), __fmul_rn(b.w, sn.w));
            hi4.x = __fadd_rn(__fmul_rn(b.x, c.x), __fmul_rn(a.x, sn.x));
            hi4.y = __fadd_rn(__fmul_rn(b.y, c.y), __fmul_rn(a.y, sn.y));
            hi4.z = __fadd_rn(__fmul_rn(b.z, c.z), __fmul_rn(a.z, sn.z));
            hi4.w = __fadd_rn(__fmul_rn(b.w, c.w), __fmul_rn(a.w, sn.w));
            *reinterpret_cast<float4 *>(kt + r * KS + d) = lo4;
            *reinterpret_cast<float4 *>(kt + r * KS + H + d) = hi4;
        }
        __syncthreads();
        // Scores: one (head, key) per thread, sequential FMA over dim.
        for (uint32_t i = threadIdx.x; i < G * rows; i += kDecThreads) {
            const uint32_t g = i / rows, r = i - g * rows;
            const float *qv = qs + g * D, *kv = kt + r * KS;
            float a = 0.0f;
#pragma unroll
            for (uint32_t d = 0; d < D; d += 4) {
                const float4 q4 = ld4(qv + d), k4 = ld4(kv + d);
                a = fmaf(q4.x, k4.x, a);
                a = fmaf(q4.y, k4.y, a);
                a = fmaf(q4.z, k4.z, a);
                a = fmaf(q4.w, k4.w, a);
            }
            sc[g * kDecTile + r] = __fmul_rn(a, scale);
        }
        __syncthreads();
        for (uint32_t g = warp; g < G; g += warps) {
            const float ninf = -__int_as_float(0x7f800000);
            const float v0 = lane < static_cast<int>(rows) ? sc[g * kDecTile + lane] : ninf;
            const float v1 = lane + 32 < static_cast<int>(rows) ? sc[g * kDecTile + lane + 32] : ninf;
            const float m = fmaxf(mrow[g], warp_max(fmaxf(v0, v1)));
            const float e0 = lane < static_cast<int>(rows) ? plamo_exp(__fsub_rn(v0, m)) : 0.0f;
            const float e1 = lane + 32 < static_cast<int>(rows) ? plamo_exp(__fsub_rn(v1, m)) : 0.0f;
            if (lane < static_cast<int>(rows)) sc[g * kDecTile + lane] = e0;
            if (lane + 32 < static_cast<int>(rows)) sc[g * kDecTile + lane + 32] = e1;
            const float tile_sum = warp_sum(__fadd_rn(e0, e1));
            if (lane == 0) {
                const float cr = plamo_exp(__fsub_rn(mrow[g], m));
                lrow[g] = __fadd_rn(__fmul_rn(lrow[g], cr), tile_sum);
                mrow[g] = m;
                corr[g] = cr;
            }
        }
        __syncthreads();
        for (uint32_t i = threadIdx.x; i < G * 32; i += kDecThreads) {
            const uint32_t g = i >> 5, d = (i & 31) * 4;
            float4 a = ld4(acc + g * D + d);
            const float cr = corr[g];
            a = make_float4(__fmul_rn(a.x, cr), __fmul_rn(a.y, cr), __fmul_rn(a.z, cr), __fmul_rn(a.w, cr));
            const float *sg = sc + g * kDecTile;
#pragma unroll 8
            for (uint32_t r = 0; r < rows; ++r) {
                const float pr = sg[r];
                const float4 v4 = ld4(vt + r * D + d);
                a.x = fmaf(pr, v4.x, a.x);
                a.y = fmaf(pr, v4.y, a.y);
                a.z = fmaf(pr, v4.z, a.z);
                a.w = fmaf(pr, v4.w, a.w);
            }
            *reinterpret_cast<float4 *>(acc + g * D + d) = a;
        }
        __syncthreads();
        const uint64_t next = base + kDecTile;
        if (next < k1) stage(next, static_cast<uint32_t>(k1 - next < kDecTile ? k1 - next : kDecTile));
    }
    __syncthreads();

    // Every cluster rank merges its share of the group's outputs from all
    // splits' partials (distributed shared memory, fixed split order).
    cluster.sync();
    {
        float *w = kt;  // [G][S] weights, then [G] denominators
        // One (head, split) pair per lane, a head's S splits on S consecutive
        // lanes of one warp: the max over splits by shuffles, one exp each,
        // then the denominator as the same in-order FMA chain over splits.
        for (uint32_t t0 = static_cast<uint32_t>(warp) * 32; t0 < G * S; t0 += warps * 32) {
            const uint32_t t = t0 + lane, g = t / S, r = t % S;
            const bool valid = t < G * S;
            const float m = valid ? cluster.map_shared_rank(mrow, r)[g] : -__int_as_float(0x7f800000);
            const float l = valid ? cluster.map_shared_rank(lrow, r)[g] : 0.0f;
            float M = m;
#pragma unroll
            for (int o = S / 2; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
            const float e = plamo_exp(__fsub_rn(m, M));
            if (valid) w[g * S + r] = e;
            float Ls = 0.0f;
#pragma unroll
            for (int q = 0; q < S; ++q) {
                const int src = static_cast<int>((lane & ~static_cast<uint32_t>(S - 1)) + q);
                Ls = fmaf(__shfl_sync(0xffffffffu, l, src), __shfl_sync(0xffffffffu, e, src), Ls);
            }
            if (valid && r == 0) w[G * S + g] = Ls;
        }
        __syncthreads();
        const uint32_t per = (G * D + S - 1) / S, i0 = cluster.block_rank() * per;
        const uint32_t i1 = min(i0 + per, G * D);
        for (uint32_t i = i0 + threadIdx.x; i < i1; i += kDecThreads) {
            const uint32_t g = i / D;
            float parts[S];
#pragma unroll
            for (int r = 0; r < S; ++r) parts[r] = cluster.map_shared_rank(acc, r)[i];
            float A = 0.0f;
#pragma unroll
            for (int r = 0; r < S; ++r) A = fmaf(parts[r], w[g * S + r], A);
            p.out[static_cast<uint64_t>(kh * G) * D + i] = __fdiv_rn(A, w[G * S + g]);
        }
    }
    cluster.sync();
    if (p.trace && threadIdx.x == 0) {
        const uint64_t t = global_ns();
        trace_stamp(p.trace, 2, t);
        trace_stamp(p.trace, 3, t);
    }
}

__global__ void __cluster_dims__(1, kDec128Splits, 1) __launch_bounds__(kDecThreads)
    decode_attention128_kernel(DecodeAttnParams p) {
    decode_attention128_body<kDec128Splits>(p);
}

// Several independent requests in one launch (blockIdx.z = request): each
// has its own KV rings, counter and projection row.
__global__ void __cluster_dims__(1, kDec128BatchSplits, 1) __launch_bounds__(kDecThreads)
    decode_attention128_batch_kernel(const DecodeAttnParams *ps) {
    decode_attention128_body<kDec128BatchSplits>(ps[blockIdx.z]);
}

// DT: compile-time head dim (128) for the vectorised path, 0 for any even dim.
template <int DT>
__global__ void __cluster_dims__(1, kDecSplits, 1) __launch_bounds__(kDecThreads)
    decode_attention_kernel(DecodeAttnParams p) {
    extern __shared__ __align__(16) float sm[];
    const uint32_t D = DT ? DT : p.dim, half = D / 2, G = p.qh / p.kh, KS = decode_key_stride(D);
    const uint32_t kh = blockIdx.x, split = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = kDecThreads / 32;
    float *qs = sm;
    float *kt = qs + G * D;
    float *vt = kt + kDecTile * KS;
    float *sc = vt + kDecTile * D;
    float *acc = sc + G * kDecTile;
    float *knew = acc + G * D;
    float *vnew = knew + D;
    float *mrow = vnew + D;
    float *lrow = mrow + G;
    float *corr = lrow + G;
    cooperative_groups::cluster_group cluster = cooperative_groups::this_cluster();

    pdl_wait();
    const uint64_t P = *p.L.appended;
    const uint64_t lo = window_start(p.L, P, 0);
    const uint32_t n = static_cast<uint32_t>(P + 1 - lo);
    const uint64_t k0 = lo + static_cast<uint64_t>(n) * split / kDecSplits;
    const uint64_t k1 = lo + static_cast<uint64_t>(n) * (split + 1) / kDecSplits;
    const float *table_q = p.L.table + static_cast<uint64_t>(n - 1) * D;

    // Q heads of the group: RMSNorm(+1), rotate at the query position.
    for (uint32_t g = warp; g < G; g += warps) {
        const float *x = p.qkv + static_cast<uint64_t>(kh * G + g) * D;
        float ss = 0.0f;
        if constexpr (DT != 0) {
#pragma unroll
            for (uint32_t i = lane; i < DT; i += 32) ss += x[i] * x[i];
        } else {
            for (uint32_t i = lane; i < D; i += 32) ss += x[i] * x[i];
        }
        const float inv = rms_inverse(warp_sum(ss), D);
        for (uint32_t i = lane; i < half; i += 32) {
            const float a = rms_apply(x[i], inv, p.L.qn[i], 1.0f);
            const float b = rms_apply(x[i + half], inv, p.L.qn[i + half], 1.0f);
            const float c = table_q[i], s = table_q[half + i];
            qs[g * D + i] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
            qs[g * D + i + half] = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
        }
    }
    // The new row: normalised K (unrotated) and V, stored to the ring by the
    // CTA whose split contains it.
    const bool has_new = k1 == P + 1;
    if (has_new && warp == warps - 1) {
        const float *x = p.qkv + static_cast<uint64_t>(p.qh + kh) * D;
        const float *v = p.qkv + static_cast<uint64_t>(p.qh + p.kh + kh) * D;
        float ss = 0.0f;
        for (uint32_t i = lane; i < D; i += 32) ss += x[i] * x[i];
        const float inv = rms_inverse(warp_sum(ss), D);
        float *const kdst = kv_key(p.L, P) + kh * D, *const vdst = kv_value(p.L, P) + kh * D;
        for (uint32_t i = lane; i < D; i += 32) {
            const float k = rms_apply(x[i], inv, p.L.kn[i], 1.0f);
            knew[i] = k;
            vnew[i] = v[i];
            kdst[i] = k;
            vdst[i] = v[i];
        }
    }
    for (uint32_t i = threadIdx.x; i < G * D; i += kDecThreads) acc[i] = 0.0f;
    for (uint32_t g = threadIdx.x; g < G; g += kDecThreads) {
        mrow[g] = -__int_as_float(0x7f800000);
        lrow[g] = 0.0f;
    }
    __syncthreads();

    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(D)));
    for (uint64_t base = k0; base < k1; base += kDecTile) {
        const uint32_t rows = static_cast<uint32_t>(k1 - base < kDecTile ? k1 - base : kDecTile);
        if constexpr (DT != 0) {
            // 4 coordinate pairs per item, float4 loads and stores.
            constexpr uint32_t Q = DT / 8;  // float4 groups per half
            const uint32_t items = rows * Q;
            for (uint32_t i0 = threadIdx.x; i0 < items; i0 += 2 * kDecThreads) {
                float4 a[2], b[2], c[2], sn[2], va[2], vb[2];
                uint32_t rr[2], dd[2];
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const uint32_t i = i0 + u * kDecThreads;
                    rr[u] = dd[u] = 0;
                    if (i < items) {
                        const uint32_t r = i / Q, d = (i - r * Q) * 4;
                        const uint64_t key = base + r;
                        const float *ksrc, *vsrc;
                        if (key < P) {
                            ksrc = kv_key(p.L, key) + kh * DT;
                            vsrc = kv_value(p.L, key) + kh * DT;
                        } else {
                            ksrc = knew;
                            vsrc = vnew;
                        }
                        const float *cs = p.L.table + (key - lo) * DT;
                        a[u] = ld4(ksrc + d);
                        b[u] = ld4(ksrc + d + DT / 2);
                        c[u] = ld4(cs + d);
                        sn[u] = ld4(cs + DT / 2 + d);
                        va[u] = ld4(vsrc + d);
                        vb[u] = ld4(vsrc + d + DT / 2);
                        rr[u] = r;
                        dd[u] = d;
                    }
                }
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    if (i0 + u * kDecThreads < items) {
                        const uint32_t r = rr[u], d = dd[u];
                        float4 lo4, hi4;
                        lo4.x = __fsub_rn(__fmul_rn(a[u].x, c[u].x), __fmul_rn(b[u].x, sn[u].x));
                        lo4.y = __fsub_rn(__fmul_rn(a[u].y, c[u].y), __fmul_rn(b[u].y, sn[u].y));
                        lo4.z = __fsub_rn(__fmul_rn(a[u].z, c[u].z), __fmul_rn(b[u].z, sn[u].z));
                        lo4.w = __fsub_rn(__fmul_rn(a[u].w, c[u].w), __fmul_rn(b[u].w, sn[u].w));
                        hi4.x = __fadd_rn(__fmul_rn(b[u].x, c[u].x), __fmul_rn(a[u].x, sn[u].x));
                        hi4.y = __fadd_rn(__fmul_rn(b[u].y, c[u].y), __fmul_rn(a[u].y, sn[u].y));
                        hi4.z = __fadd_rn(__fmul_rn(b[u].z, c[u].z), __fmul_rn(a[u].z, sn[u].z));
                        hi4.w = __fadd_rn(__fmul_rn(b[u].w, c[u].w), __fmul_rn(a[u].w, sn[u].w));
                        *reinterpret_cast<float4 *>(kt + r * KS + d) = lo4;
                        *reinterpret_cast<float4 *>(kt + r * KS + d + DT / 2) = hi4;
                        *reinterpret_cast<float4 *>(vt + r * DT + d) = va[u];
                        *reinterpret_cast<float4 *>(vt + r * DT + d + DT / 2) = vb[u];
                    }
                }
            }
        } else {
            const uint32_t items = rows * half;
            for (uint32_t i = threadIdx.x; i < items; i += kDecThreads) {
                const uint32_t r = i / half, d = i - r * half;
                const uint64_t key = base + r;
                const float *ksrc, *vsrc;
                if (key < P) {
                    ksrc = kv_key(p.L, key) + kh * D;
                    vsrc = kv_value(p.L, key) + kh * D;
                } else {
                    ksrc = knew;
                    vsrc = vnew;
                }
                const float *cs = p.L.table + (key - lo) * D;
                const float a = ksrc[d], b = ksrc[d + half], c = cs[d], sn = cs[half + d];
                kt[r * KS + d] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, sn));
                kt[r * KS + d + half] = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, sn));
                vt[r * D + d] = vsrc[d];
                vt[r * D + d + half] = vsrc[d + half];
            }
        }
        __syncthreads();
        // Scores: one (head, key) per thread, sequential FMA over dim.
        for (uint32_t i = threadIdx.x; i < G * rows; i += kDecThreads) {
            const uint32_t g = i / rows, r = i - g * rows;
            const float *qv = qs + g * D, *kv = kt + r * KS;
            float a = 0.0f;
            if constexpr (DT != 0) {
#pragma unroll
                for (uint32_t d = 0; d < DT; d += 4) {
                    const float4 q4 = ld4(qv + d), k4 = ld4(kv + d);
                    a = fmaf(q4.x, k4.x, a);
                    a = fmaf(q4.y, k4.y, a);
                    a = fmaf(q4.z, k4.z, a);
                    a = fmaf(q4.w, k4.w, a);
                }
            } else {
                for (uint32_t d = 0; d < D; ++d) a = fmaf(qv[d], kv[d], a);
            }
            sc[g * kDecTile + r] = __fmul_rn(a, scale);
        }
        __syncthreads();
        // Online softmax: one warp per head, two keys per lane.
        for (uint32_t g = warp; g < G; g += warps) {
            const float ninf = -__int_as_float(0x7f800000);
            const float v0 = lane < static_cast<int>(rows) ? sc[g * kDecTile + lane] : ninf;
            const float v1 = lane + 32 < static_cast<int>(rows) ? sc[g * kDecTile + lane + 32] : ninf;
            const float m = fmaxf(mrow[g], warp_max(fmaxf(v0, v1)));
            const float e0 = lane < static_cast<int>(rows) ? plamo_exp(__fsub_rn(v0, m)) : 0.0f;
            const float e1 = lane + 32 < static_cast<int>(rows) ? plamo_exp(__fsub_rn(v1, m)) : 0.0f;
            if (lane < static_cast<int>(rows)) sc[g * kDecTile + lane] = e0;
            if (lane + 32 < static_cast<int>(rows)) sc[g * kDecTile + lane + 32] = e1;
            const float tile_sum = warp_sum(__fadd_rn(e0, e1));
            if (lane == 0) {
                const float cr = plamo_exp(__fsub_rn(mrow[g], m));
                lrow[g] = __fadd_rn(__fmul_rn(lrow[g], cr), tile_sum);
                mrow[g] = m;
                corr[g] = cr;
            }
        }
        __syncthreads();
        // Weighted values: sequential FMA over the tile's keys.
        if constexpr (DT != 0) {
            for (uint32_t i = threadIdx.x; i < G * (DT / 4); i += kDecThreads) {
                const uint32_t g = i / (DT / 4), d = (i - g * (DT / 4)) * 4;
                float4 a = ld4(acc + g * DT + d);
                const float cr = corr[g];
                a = make_float4(__fmul_rn(a.x, cr), __fmul_rn(a.y, cr), __fmul_rn(a.z, cr), __fmul_rn(a.w, cr));
                const float *sg = sc + g * kDecTile;
#pragma unroll 8
                for (uint32_t r = 0; r < rows; ++r) {
                    const float pr = sg[r];
                    const float4 v4 = ld4(vt + r * DT + d);
                    a.x = fmaf(pr, v4.x, a.x);
                    a.y = fmaf(pr, v4.y, a.y);
                    a.z = fmaf(pr, v4.z, a.z);
                    a.w = fmaf(pr, v4.w, a.w);
                }
                *reinterpret_cast<float4 *>(acc + g * DT + d) = a;
            }
        } else {
            for (uint32_t i = threadIdx.x; i < G * D; i += kDecThreads) {
                const uint32_t g = i / D, d = i - g * D;
                float a = __fmul_rn(acc[i], corr[g]);
                for (uint32_t r = 0; r < rows; ++r) a = fmaf(sc[g * kDecTile + r], vt[r * D + d], a);
                acc[i] = a;
            }
        }
        __syncthreads();
    }

    // Merge the cluster's partials on rank 0 through distributed shared
    // memory, in split order: M = max m_s, L = sum l_s e^(m_s - M),
    // out = sum acc_s e^(m_s - M) / L.
    cluster.sync();
    if (cluster.block_rank() == 0) {
        float *w = kt;  // [G][splits] weights, then [G] denominators
        if (threadIdx.x < G) {
            const uint32_t g = threadIdx.x;
            float ms[kDecSplits];
            float M = -__int_as_float(0x7f800000);
#pragma unroll
            for (int r = 0; r < kDecSplits; ++r) {
                ms[r] = cluster.map_shared_rank(mrow, r)[g];
                M = fmaxf(M, ms[r]);
            }
            float Ls = 0.0f;
#pragma unroll
            for (int r = 0; r < kDecSplits; ++r) {
                const float e = plamo_exp(__fsub_rn(ms[r], M));
                w[g * kDecSplits + r] = e;
                Ls = fmaf(cluster.map_shared_rank(lrow, r)[g], e, Ls);
            }
            w[G * kDecSplits + g] = Ls;
        }
        __syncthreads();
        for (uint32_t i = threadIdx.x; i < G * D; i += kDecThreads) {
            const uint32_t g = i / D;
            float parts[kDecSplits];
#pragma unroll
            for (int r = 0; r < kDecSplits; ++r) parts[r] = cluster.map_shared_rank(acc, r)[i];
            float A = 0.0f;
#pragma unroll
            for (int r = 0; r < kDecSplits; ++r) A = fmaf(parts[r], w[g * kDecSplits + r], A);
            p.out[static_cast<uint64_t>(kh * G) * D + i] = __fdiv_rn(A, w[G * kDecSplits + g]);
        }
    }
    pdl_launch_dependents();
    cluster.sync();  // keep every CTA's shared memory alive until rank 0 is done
}

// Store the K/V rows of tokens [first, tokens) (normalised K, V from the QKV
// buffer) into ring slots (P + t) % ring. One CTA per token.
__global__ void kv_store_kernel(AttnLayer L, AttnShape S, const float *qkv, uint64_t first) {
    pdl_wait();
    const uint64_t t = first + blockIdx.x;
    const uint64_t P = *L.appended;
    const uint64_t kvw = S.kh * S.dim;
    const float *row = qkv + t * S.qkv_stride;
    float *const kdst = kv_key(L, P + t), *const vdst = kv_value(L, P + t);
    for (uint64_t i = threadIdx.x; i < kvw; i += blockDim.x) {
        kdst[i] = row[S.qh * S.dim + i];
        vdst[i] = row[(S.qh + S.kh) * S.dim + i];
    }
    pdl_launch_dependents();
}

// Copy K/V rows of one candidate (kept per layer by a verification) to the
// ring slot of the next committed row.
__global__ void kv_commit_kernel(AttnLayer L, uint64_t kvw, const float *k_row, const float *v_row) {
    const uint64_t P = *L.appended;
    float *const kdst = kv_key(L, P), *const vdst = kv_value(L, P);
    for (uint64_t i = threadIdx.x; i < kvw; i += blockDim.x) {
        kdst[i] = k_row[i];
        vdst[i] = v_row[i];
    }
}

// Move every layer's committed-row counter back by `rows` (speculative
// rollback; the rings keep the rows, so nothing else changes).
__global__ void rollback_kernel(uint64_t *appended, uint64_t layers, uint64_t rows) {
    pdl_wait();
    for (uint64_t i = threadIdx.x; i < layers; i += blockDim.x) appended[i] -= rows;
}

// Advance every layer's committed-row counter by `rows` (end of a step).
__global__ void advance_kernel(uint64_t *appended, uint64_t layers, uint64_t rows) {
    pdl_wait();
    for (uint64_t i = threadIdx.x; i < layers; i += blockDim.x) appended[i] += rows;
}

// Host view of a ring: rows [P - count, P) into token-major arrays, keys
// also rotated at local positions 0..count-1 (the reference's rotation.out).
__global__ void kv_gather_kernel(AttnLayer L, uint64_t kvw, uint64_t heads, uint64_t dim,
                                 uint64_t count, float *k_out, float *v_out, float *rot_out) {
    const uint64_t r = blockIdx.x;
    const uint64_t P = *L.appended;
    const float *const krow = kv_key(L, P - count + r), *const vrow = kv_value(L, P - count + r);
    const uint64_t half = dim / 2;
    const float *c = L.table + r * dim, *s = c + half;
    for (uint64_t i = threadIdx.x; i < kvw; i += blockDim.x) {
        k_out[r * kvw + i] = krow[i];
        v_out[r * kvw + i] = vrow[i];
    }
    for (uint64_t i = threadIdx.x; i < heads * half; i += blockDim.x) {
        const uint64_t h = i / half, d = i % half;
        const float a = krow[h * dim + d], b = krow[h * dim + d + half];
        rot_out[r * kvw + h * dim + d] = __fsub_rn(__fmul_rn(a, c[d]), __fmul_rn(b, s[d]));
        rot_out[r * kvw + h * dim + d + half] = __fadd_rn(__fmul_rn(b, c[d]), __fmul_rn(a, s[d]));
    }
}

}  // namespace plamo
