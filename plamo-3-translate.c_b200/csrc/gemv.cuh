// Decode projections: BF16 weight x FP32 vector, FP32 accumulation.
//
// Replaces the reference's decode matvec (reference src/math.s:5-344 on the
// CPU, runtime/kernels.metal:206-252 on the GPU). Batch-1 decode streams every
// weight byte once per token, so this kernel is bound by HBM bandwidth:
//   * each CTA owns a contiguous range of output rows (balanced to one row
//     across the grid); its warps walk (row, column segment) work items, so
//     the CTA stays busy to the end whatever the row count;
//   * every lane issues 128-bit streaming loads (L1 bypass, L2 evict-first),
//     U loads per work item, double-buffered in registers so the next item's
//     weights are in flight while the current one is reduced;
//   * the input vector lives in shared memory as FP32, built by a prologue
//     that also fuses the RMSNorms and the residual update that precede the
//     projection in a PLaMo-3 layer (each CTA recomputes the same normalised
//     vector; block 0 publishes the updated state);
//   * per-segment partial sums are reduced in a fixed order, then an
//     epilogue stores, applies SwiGLU to gate/up row pairs, or forms
//     per-block argmax candidates for the LM head;
//   * the first work item's weights are requested before griddepcontrol.wait,
//     so under programmatic dependent launch the weight stream of this
//     projection overlaps the tail of the previous kernel.
#pragma once
#include "common.cuh"
#include "tp.cuh"

namespace plamo {

// PRO_RESID_NORM_TP: PRO_RESID_NORM whose branch is the rank-ordered sum of a
// tensor-parallel point's partials (a separate instantiation, so the
// single-GPU kernels carry no exchange code).
enum GemvPrologue { PRO_X = 0, PRO_NORM = 1, PRO_RESID_NORM = 2, PRO_EMBED_NORM = 3, PRO_RESID_NORM_TP = 4 };
enum GemvEpilogue { EPI_STORE = 0, EPI_SWIGLU = 1, EPI_ARGMAX = 2 };

struct GemvParams {
    const uint16_t *w;  // [rows, cols] row-major BF16
    uint64_t rows, cols;
    const float *x;               // PRO_X: input vector [cols]
    const float *state_in;        // PRO_NORM / PRO_RESID_NORM: hidden state [cols]
    const float *branch;          // PRO_RESID_NORM: branch added after its own norm
    const uint16_t *embedding;    // PRO_EMBED_NORM: BF16 table [vocab, cols]
    const uint32_t *token;        // PRO_EMBED_NORM: device token id
    uint64_t vocab;
    const uint16_t *norm1;        // branch norm weights
    float off1;
    const uint16_t *norm2;        // input norm weights
    float off2;
    float *state_out;             // block 0 writes the (updated) state here
    float *norm_out;              // block 0 writes the normalised input here
    float *y;                     // STORE/ARGMAX: [rows]; SWIGLU: [rows/2]
    float *arg_val;               // ARGMAX: per-block best value
    float *arg_val2;              // ARGMAX: per-block runner-up value (any other index)
    uint32_t *arg_idx;            // ARGMAX: per-block best index
    uint32_t *arg_nan;            // ARGMAX: per-block NaN flag
    uint32_t *error;              // set to nonzero on an invalid token
    // Tensor parallelism: role 1 = the prologue's branch is the rank-ordered
    // sum of the point's partials (PRO_RESID_NORM_TP); role 2 = the STORE
    // epilogue pushes its rows into every rank's slot of the point.
    int tp_role;
    TpPoint tp;
    unsigned long long *trace;  // launch timeline record (trace_stamp), or null
};

constexpr int kGemvThreads = 512;
constexpr int kGemvWarps = kGemvThreads / 32;

// 8 BF16 weights . 8 FP32 inputs, accumulated with explicit FMAs.
__device__ __forceinline__ float dot8(uint4 w, const float *x, float acc) {
    const float4 a = *reinterpret_cast<const float4 *>(x);
    const float4 b = *reinterpret_cast<const float4 *>(x + 4);
    acc = fmaf(bf16_lo(w.x), a.x, acc);
    acc = fmaf(bf16_hi(w.x), a.y, acc);
    acc = fmaf(bf16_lo(w.y), a.z, acc);
    acc = fmaf(bf16_hi(w.y), a.w, acc);
    acc = fmaf(bf16_lo(w.z), b.x, acc);
    acc = fmaf(bf16_hi(w.z), b.y, acc);
    acc = fmaf(bf16_lo(w.w), b.z, acc);
    acc = fmaf(bf16_hi(w.w), b.w, acc);
    return acc;
}

// Same with the 8 inputs in registers.
__device__ __forceinline__ float dot8r(uint4 w, const float *x, float acc) {
    acc = fmaf(bf16_lo(w.x), x[0], acc);
    acc = fmaf(bf16_hi(w.x), x[1], acc);
    acc = fmaf(bf16_lo(w.y), x[2], acc);
    acc = fmaf(bf16_hi(w.y), x[3], acc);
    acc = fmaf(bf16_lo(w.z), x[4], acc);
    acc = fmaf(bf16_hi(w.z), x[5], acc);
    acc = fmaf(bf16_lo(w.w), x[6], acc);
    acc = fmaf(bf16_hi(w.w), x[7], acc);
    return acc;
}

// Build the FP32 input vector in shared memory. All blocks compute the same
// bits (same reduction shape), block 0 publishes state/normalised copies.
//
// Latency matters more than work here (a few KB per block while the weight
// stream waits), so every global load of a phase is issued before any of
// them is used: the vector path keeps up to kPV float4 per thread in
// registers, one L2 round trip per input instead of one per loop trip.
constexpr int kPV = 4;

// The vector path's norm weights, loaded before the dependency wait: they
// are constants of the model, so their latency overlaps the previous kernel.
struct NormWeights {
    uint2 w1[kPV], w2[kPV];
};

template <int PRO>
__device__ __forceinline__ void gemv_norm_weights(const GemvParams &p, NormWeights &nw) {
    constexpr bool kResid = PRO == PRO_RESID_NORM || PRO == PRO_RESID_NORM_TP;
    if constexpr (PRO == PRO_X || PRO == PRO_EMBED_NORM) {
        return;
    } else {
        const uint32_t nt = blockDim.x;
        if (p.cols % 4 != 0 || p.cols > 4ull * kPV * nt) return;
        const uint32_t n4 = static_cast<uint32_t>(p.cols / 4);
#pragma unroll
        for (int k = 0; k < kPV; ++k) {
            const uint32_t i = threadIdx.x + k * nt;
            if (i < n4) {
                if (kResid) nw.w1[k] = *reinterpret_cast<const uint2 *>(p.norm1 + 4 * i);
                nw.w2[k] = *reinterpret_cast<const uint2 *>(p.norm2 + 4 * i);
            }
        }
    }
}

template <int PRO>
__device__ __forceinline__ bool gemv_prologue(const GemvParams &p, float *xs, float *red, const NormWeights &nw) {
    constexpr bool kResid = PRO == PRO_RESID_NORM || PRO == PRO_RESID_NORM_TP;
    constexpr bool reduce = PRO == PRO_RESID_NORM_TP;
    const uint64_t n = p.cols;
    const bool publish = blockIdx.x == 0;
    const uint32_t nt = blockDim.x;
    if (PRO == PRO_X) {
        const uint32_t n4 = static_cast<uint32_t>(n / 4);
        const float4 *x4 = reinterpret_cast<const float4 *>(p.x);
        float4 *xs4 = reinterpret_cast<float4 *>(xs);
        uint32_t i = threadIdx.x;
        for (; i + 3 * nt < n4; i += 4 * nt) {
            const float4 a = x4[i], b = x4[i + nt], c = x4[i + 2 * nt], d = x4[i + 3 * nt];
            xs4[i] = a;
            xs4[i + nt] = b;
            xs4[i + 2 * nt] = c;
            xs4[i + 3 * nt] = d;
        }
        for (; i < n4; i += nt) xs4[i] = x4[i];
        for (uint64_t j = 4ull * n4 + threadIdx.x; j < n; j += nt) xs[j] = p.x[j];
        return true;
    }
    const bool vec = n % 4 == 0 && n <= 4ull * kPV * nt;
    if (PRO == PRO_EMBED_NORM) {
        const uint32_t token = *p.token;
        if (token >= p.vocab) {
            if (publish && threadIdx.x == 0) *p.error = 1;
            return false;
        }
        const uint16_t *row = p.embedding + static_cast<uint64_t>(token) * n;
        for (uint64_t i = threadIdx.x; i < n; i += nt) xs[i] = bf16_to_f32(row[i]);
    } else if (vec) {
        const uint32_t n4 = static_cast<uint32_t>(n / 4);
        float4 st[kPV], br[kPV];
        const uint32_t tag = reduce && p.tp.ll ? *p.tp.epoch + 1 : 0;
        if (reduce && !p.tp.ll) {
            if (threadIdx.x == 0) tp_wait_flags(p.tp);
            __syncthreads();
        }
        if (reduce && p.tp.ll) tp_ll_sum_groups<kPV>(p.tp, threadIdx.x, nt, n4, tag, br);
#pragma unroll
        for (int k = 0; k < kPV; ++k) {
            const uint32_t i = threadIdx.x + k * nt;
            if (i < n4) {
                st[k] = ld4(p.state_in + 4 * i);
                if (kResid) {
                    if (!reduce) br[k] = ld4(p.branch + 4 * i);
                    else if (!p.tp.ll) br[k] = tp_sum4(p.tp, 4 * i);
                }
            }
        }
        if (kResid) {
            float s = 0.0f;
#pragma unroll
            for (int k = 0; k < kPV; ++k)
                if (threadIdx.x + k * nt < n4) s += sq4(br[k]);
            const float inv = rms_inverse(block_sum(s, red), n);
#pragma unroll
            for (int k = 0; k < kPV; ++k) {
                const uint32_t i = threadIdx.x + k * nt;
                if (i < n4) {
                    const float4 b = apply4(br[k], inv, norm4(nw.w1[k], p.off1));
                    st[k] = make_float4(__fadd_rn(st[k].x, b.x), __fadd_rn(st[k].y, b.y),
                                        __fadd_rn(st[k].z, b.z), __fadd_rn(st[k].w, b.w));
                }
            }
        }
        float s = 0.0f;
#pragma unroll
        for (int k = 0; k < kPV; ++k) {
            const uint32_t i = threadIdx.x + k * nt;
            if (i < n4) {
                s += sq4(st[k]);
                if (publish && p.state_out) *reinterpret_cast<float4 *>(p.state_out + 4 * i) = st[k];
            }
        }
        const float inv = rms_inverse(block_sum(s, red), n);
#pragma unroll
        for (int k = 0; k < kPV; ++k) {
            const uint32_t i = threadIdx.x + k * nt;
            if (i < n4) {
                const float4 v = apply4(st[k], inv, norm4(nw.w2[k], p.off2));
                *reinterpret_cast<float4 *>(xs + 4 * i) = v;
                if (publish && p.norm_out) *reinterpret_cast<float4 *>(p.norm_out + 4 * i) = v;
            }
        }
        return true;
    } else if (PRO == PRO_NORM) {
        for (uint64_t i = threadIdx.x; i < n; i += nt) xs[i] = p.state_in[i];
    } else {  // PRO_RESID_NORM(_TP), any length: state + rmsnorm(branch, norm1, off1)
        const uint32_t tag = reduce && p.tp.ll ? *p.tp.epoch + 1 : 0;
        if (reduce && !p.tp.ll) {
            if (threadIdx.x == 0) tp_wait_flags(p.tp);
            __syncthreads();
        }
        float s = 0.0f;
        for (uint64_t i = threadIdx.x; i < n; i += nt) {
            const float b = !reduce ? p.branch[i] : p.tp.ll ? tp_ll_sum1(p.tp, i, tag) : tp_sum1(p.tp, i);
            s += b * b;
        }
        const float inv = rms_inverse(block_sum(s, red), n);
        for (uint64_t i = threadIdx.x; i < n; i += nt) {
            const float b = !reduce ? p.branch[i] : p.tp.ll ? tp_ll_sum1(p.tp, i, tag) : tp_sum1(p.tp, i);
            xs[i] = __fadd_rn(p.state_in[i], rms_apply(b, inv, p.norm1[i], p.off1));
        }
    }
    __syncthreads();
    float s = 0.0f;
    for (uint64_t i = threadIdx.x; i < n; i += nt) {
        const float v = xs[i];
        s += v * v;
        if (publish && p.state_out) p.state_out[i] = v;
    }
    const float inv = rms_inverse(block_sum(s, red), n);
    for (uint64_t i = threadIdx.x; i < n; i += nt) {
        const float v = rms_apply(xs[i], inv, p.norm2[i], p.off2);
        xs[i] = v;
        if (publish && p.norm_out) p.norm_out[i] = v;
    }
    return true;
}

// Argmax candidate order: larger value first, then lower index.
__device__ __forceinline__ bool arg_better(float v, uint32_t i, float bv, uint32_t bi) {
    return v > bv || (v == bv && i < bi);
}

// Fold candidate (v, i, v2: its own runner-up) into (bv, bi, sv): the best of
// the two stays best; the runner-up is the largest value of any other index.
__device__ __forceinline__ void top2_merge(float v, uint32_t i, float v2, float &bv, uint32_t &bi, float &sv) {
    if (arg_better(v, i, bv, bi)) {
        sv = fmaxf(fmaxf(sv, v2), bv);
        bv = v;
        bi = i;
    } else {
        sv = fmaxf(sv, fmaxf(v, v2));
    }
}

// Fixed-order reduction of per-slot partials ([unit][slot][pair]), then the
// epilogue: store, SwiGLU of gate/up pairs, or per-block argmax candidates.
template <int EPI>
__device__ __forceinline__ void gemv_epilogue(const GemvParams &p, const float *partial, uint64_t u0,
                                              uint64_t u1, uint64_t slots, float *) {
    __shared__ float best_val[32];
    __shared__ uint32_t best_idx[32];
    __shared__ uint32_t any_nan;
    constexpr int kPair = EPI == EPI_SWIGLU ? 2 : 1;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int warps = (blockDim.x + 31) >> 5;
    float bv = -__int_as_float(0x7f800000), sv = bv;
    uint32_t bi = 0xffffffffu;
    bool saw_nan = false;
    const uint32_t ll_tag = EPI == EPI_STORE && p.tp_role == 2 && p.tp.ll ? *p.tp.epoch + 1 : 0;
    for (uint64_t u = threadIdx.x; u < u1 - u0; u += blockDim.x) {
        float t0 = 0.0f, t1 = 0.0f;
        for (uint64_t s = 0; s < slots; ++s) {
            t0 += partial[(u * slots + s) * kPair];
            if (kPair == 2) t1 += partial[(u * slots + s) * kPair + 1];
        }
        const uint64_t unit = u0 + u;
        if (EPI == EPI_SWIGLU) {
            p.y[unit] = swiglu(t0, t1);
        } else if (EPI == EPI_STORE && p.tp_role == 2) {
            if (tp_failed(p.tp.error)) continue;
            if (p.tp.ll) tp_ll_store(p.tp, unit, t0, ll_tag);
            else
                for (uint32_t r = 0; r < p.tp.tp; ++r) p.tp.peer_parts[r][unit] = t0;
        } else {
            p.y[unit] = t0;
            if (EPI == EPI_ARGMAX) {
                if (t0 != t0) saw_nan = true;
                else top2_merge(t0, static_cast<uint32_t>(unit), -__int_as_float(0x7f800000), bv, bi, sv);
            }
        }
    }
    if (EPI == EPI_STORE && p.tp_role == 2 && !p.tp.ll) tp_signal(p.tp);
    if (EPI == EPI_ARGMAX) {
        __shared__ float second_val[32];
        if (threadIdx.x == 0) any_nan = 0;
        __syncthreads();
        if (saw_nan) any_nan = 1;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
            const float os = __shfl_xor_sync(0xffffffffu, sv, o);
            top2_merge(ov, oi, os, bv, bi, sv);
        }
        if (lane == 0) {
            best_val[warp] = bv;
            best_idx[warp] = bi;
            second_val[warp] = sv;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            for (int w = 1; w < warps; ++w) top2_merge(best_val[w], best_idx[w], second_val[w], bv, bi, sv);
            p.arg_val[blockIdx.x] = bv;
            p.arg_idx[blockIdx.x] = bi;
            p.arg_nan[blockIdx.x] = any_nan;
            if (p.arg_val2) p.arg_val2[blockIdx.x] = sv;
        }
    }
}

// Register-streamed variant for shapes the bulk kernel does not take.
// U: 256-column chunks per work item (U = 0: any shape, scalar loads).
template <int PRO, int EPI, int U>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(GemvParams p) {
    extern __shared__ __align__(16) float smem[];
    __shared__ float red[kGemvWarps];

    constexpr int kPair = EPI == EPI_SWIGLU ? 2 : 1;
    const uint64_t cols = p.cols;
    const uint64_t units = p.rows / kPair;
    const uint64_t u0 = units * blockIdx.x / gridDim.x;
    const uint64_t u1 = units * (blockIdx.x + 1) / gridDim.x;
    const uint64_t seg_cols = U ? 256 * U : cols;
    const uint64_t segs = U ? cols / seg_cols : 1;
    const uint64_t items = (u1 - u0) * segs;
    const uint64_t cols_pad = (cols + 3) & ~3ull;
    float *xs = smem;
    float *partial = smem + cols_pad;  // [(u1-u0) * segs * kPair]

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint64_t policy = evict_first_policy();
    const uint64_t half_rows = p.rows / 2;

    // Row pointer of work item j, pair member m (32-bit split of j).
    const uint32_t segs32 = static_cast<uint32_t>(segs);
    auto row_ptr = [&](uint64_t j, int m) -> const uint16_t * {
        const uint32_t jj = static_cast<uint32_t>(j), q = jj / segs32;
        const uint64_t unit = u0 + q;
        const uint64_t row = m ? unit + half_rows : unit;
        return p.w + row * cols + static_cast<uint64_t>(jj - q * segs32) * seg_cols;
    };

    pdl_launch_dependents();
    constexpr int kLoads = (U ? U : 1) * kPair;
    uint4 cur[kLoads];
    uint64_t j = warp;
    if (U) {
        if (j < items) {
#pragma unroll
            for (int m = 0; m < kPair; ++m)
#pragma unroll
                for (int k = 0; k < U; ++k)
                    cur[m * U + k] = load_stream(row_ptr(j, m) + k * 256 + lane * 8, policy);
        }
    }

    NormWeights nw;
    gemv_norm_weights<PRO>(p, nw);
    pdl_wait();
    const bool ok = gemv_prologue<PRO>(p, xs, red, nw);
    __syncthreads();
    if (!ok) return;

    if (U) {
        for (; j < items; j += kGemvWarps) {
            const uint64_t jn = j + kGemvWarps;
            uint4 nxt[kLoads];
            if (jn < items) {
#pragma unroll
                for (int m = 0; m < kPair; ++m)
#pragma unroll
                    for (int k = 0; k < U; ++k)
                        nxt[m * U + k] = load_stream(row_ptr(jn, m) + k * 256 + lane * 8, policy);
            }
            const float *xseg = xs + static_cast<uint64_t>(static_cast<uint32_t>(j) % segs32) * seg_cols + lane * 8;
#pragma unroll
            for (int m = 0; m < kPair; ++m) {
                float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
                for (int k = 0; k < U; ++k) {
                    if (k & 1) a1 = dot8(cur[m * U + k], xseg + k * 256, a1);
                    else a0 = dot8(cur[m * U + k], xseg + k * 256, a0);
                }
                const float s = warp_sum(a0 + a1);
                if (lane == 0) partial[(j * kPair) + m] = s;
            }
            if (jn < items) {
#pragma unroll
                for (int k = 0; k < kLoads; ++k) cur[k] = nxt[k];
            }
        }
    } else {
        for (; j < items; j += kGemvWarps) {
#pragma unroll
            for (int m = 0; m < kPair; ++m) {
                const uint16_t *wr = row_ptr(j, m);
                float a = 0.0f;
                for (uint64_t c = lane; c < cols; c += 32) a = fmaf(bf16_to_f32(wr[c]), xs[c], a);
                a = warp_sum(a);
                if (lane == 0) partial[(j * kPair) + m] = a;
            }
        }
    }
    __syncthreads();
    gemv_epilogue<EPI>(p, partial, u0, u1, segs, red);
}

// ---------------------------------------------------------------------------
// Bulk-streamed variant (cols % 8 == 0, 16-byte aligned rows).
//
// A CTA's rows are one contiguous byte range of W (two for gate/up pairs). A
// producer warp streams it through a ring of shared-memory stages with
// cp.async.bulk (the TMA engine, plain 1-D copies), each stage guarded by a
// full/empty mbarrier pair; the first stages are requested before
// griddepcontrol.wait, so under programmatic dependent launch the stream
// starts while the previous kernel drains. A chunk is a whole number of
// rows (several short rows, or one long row), split into 512-element
// sub-ranges (the last one of a row shorter when cols % 512 != 0); consumer
// warp w takes sub-ranges w, w+16, w+32, w+48 of every chunk, which are
// always the same column slots, so each warp keeps its slice of the input
// vector in registers for the whole kernel and reduces each sub-range to one
// partial sum per (row, 512-column slot).
constexpr int kBulkConsumers = 16;
constexpr int kBulkThreads = (kBulkConsumers + 1) * 32;
constexpr int kSubElems = 512;
constexpr int kMaxStages = 12;
constexpr int kMaxSets = 4;  // sub-ranges per warp per chunk

// Column slots of a row: ceil(cols / 512).
__host__ __device__ inline uint32_t bulk_slots(uint64_t cols) {
    return static_cast<uint32_t>((cols + kSubElems - 1) / kSubElems);
}

// Sub-ranges per chunk for `slots` 512-column slots per row: a whole number
// of rows (so every chunk starts at slot 0 and each warp's column slots stay
// fixed), at most 16 * kMaxSets sub-ranges, chosen so the 16 consumer warps
// get the most even shares (10 slots: 3 rows = 30 sub-ranges, 94% of the
// warps busy instead of 10 of 16), then the smallest such chunk.
__host__ __device__ inline uint32_t bulk_chunk_subs(uint32_t slots) {
    uint32_t best = slots, best_den = 16 * ((slots + 15) / 16);
    for (uint32_t r = 2; r * slots <= 16u * kMaxSets; ++r) {
        const uint32_t subs = r * slots, den = 16 * ((subs + 15) / 16);
        if (static_cast<uint64_t>(subs) * best_den > static_cast<uint64_t>(best) * den) {
            best = subs;
            best_den = den;
        }
    }
    return best;
}

// PART: rows end inside a 512-column slot (cols % 512 != 0); the lanes past
// a row's end read nothing and contribute zero. Without it the sub-range
// addressing is the plain j * 512 of full slots.
template <int PRO, int EPI, int SETS, bool PART>
__global__ void __launch_bounds__(kBulkThreads) gemv_bulk_kernel(GemvParams p, int stages) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t full_bar[kMaxStages];
    __shared__ __align__(8) uint64_t empty_bar[kMaxStages];
    __shared__ float red[32];
    __shared__ int abort_flag;

    constexpr int kPair = EPI == EPI_SWIGLU ? 2 : 1;
    const uint64_t cols = p.cols;
    const uint64_t units = p.rows / kPair;
    const uint64_t u0 = units * blockIdx.x / gridDim.x;
    const uint64_t u1 = units * (blockIdx.x + 1) / gridDim.x;
    const uint64_t rows_local = u1 - u0;
    const uint32_t slots = PART ? bulk_slots(cols) : static_cast<uint32_t>(cols / kSubElems);
    const uint32_t csubs = bulk_chunk_subs(slots);
    const uint32_t cols32 = static_cast<uint32_t>(cols);
    // Full slots: a chunk is csubs 1 KB sub-ranges; partial: rpc rows.
    const uint32_t rpc = PART ? csubs / slots : 0;
    const uint32_t chunk_bytes = PART ? rpc * cols32 * 2 : csubs * kSubElems * 2;
    const uint32_t subs_per_range = static_cast<uint32_t>(rows_local) * slots;
    const uint32_t cpr = (subs_per_range + csubs - 1) / csubs;  // chunks per range
    const uint32_t total = kPair * cpr;
    const uint64_t cols_pad = (cols + 3) & ~3ull;
    unsigned char *ring = smem_raw;
    float *xs = reinterpret_cast<float *>(smem_raw + static_cast<size_t>(stages) * chunk_bytes);
    float *partial = xs + cols_pad;  // [rows_local][slots][kPair]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const bool producer = warp == kBulkConsumers;
    const uint64_t policy = evict_first_policy();
    const uint64_t half_rows = p.rows / 2;
    // The CTA's rows (gate rows, then the matching up rows of a pair);
    // selected, not indexed, so no local-memory array is formed.
    const uint16_t *const range_gate = p.w + u0 * cols;
    const uint16_t *const range_up = p.w + (u0 + half_rows) * cols;
    const uint64_t t_entry = p.trace ? global_ns() : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], kBulkConsumers);
        }
        abort_flag = 0;
        fence_barrier_init();
    }
    __syncthreads();
    // Let the next kernel's CTAs take SMs as soon as this grid's CTAs retire:
    // they stream their first weight stages while this grid finishes, and
    // their griddepcontrol.wait still orders every read of our results.
    pdl_launch_dependents();

    auto issue = [&](uint32_t k, uint32_t s) {
        const uint32_t m = (kPair == 2 && k >= cpr) ? 1u : 0u;
        const uint32_t kc = k - m * cpr;
        const uint32_t left = subs_per_range - kc * csubs;
        const uint32_t bytes = PART ? (left < csubs ? left : csubs) / slots * cols32 * 2
                                    : (left < csubs ? left : csubs) * kSubElems * 2;
        mbar_expect_tx(&full_bar[s], bytes);
        const uint16_t *base = m ? range_up : range_gate;
        const uint16_t *src = PART ? base + static_cast<uint64_t>(kc) * rpc * cols
                                   : base + static_cast<uint64_t>(kc) * csubs * kSubElems;
        bulk_load(ring + static_cast<size_t>(s) * chunk_bytes, src, bytes, &full_bar[s], policy);
    };
    const uint32_t primed = total < static_cast<uint32_t>(stages) ? total : static_cast<uint32_t>(stages);
    uint32_t issued = 0;  // meaningful in the producer lane only
    if (producer && lane == 0)
        for (; issued < primed; ++issued) issue(issued, issued);

    NormWeights nw;
    gemv_norm_weights<PRO>(p, nw);
    pdl_wait();
    if (p.trace && threadIdx.x == 0) trace_stamp(p.trace, 4, global_ns());
    const bool ok = gemv_prologue<PRO>(p, xs, red, nw);
    __syncthreads();
    if (p.trace && threadIdx.x == 0) {
        trace_stamp(p.trace, 0, t_entry);
        trace_stamp(p.trace, 5, t_entry);
        trace_stamp(p.trace, 1, global_ns());
    }

    // Register copy of this warp's input slots: set i serves sub-range
    // w+16i, which is row jr of a chunk at column slot js; the lane's two
    // 8-column pieces lie at col0 and col0 + 256 (zero past the row's end).
    float xr[SETS][16];
    uint32_t soff[SETS];  // PART: uint4 offset of the lane's first piece in a stage
    bool v0[SETS], v1[SETS];
    if (!producer) {
#pragma unroll
        for (int i = 0; i < SETS; ++i) {
            const uint32_t j = static_cast<uint32_t>(warp) + 16u * i;
            if constexpr (PART) {
                const uint32_t jr = j / slots, js = j - jr * slots;
                const uint32_t col0 = js * kSubElems + lane * 8;
                v0[i] = j < csubs && col0 < cols32;
                v1[i] = j < csubs && col0 + 256 < cols32;
                soff[i] = (jr * cols32 + col0) / 8;
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    xr[i][e] = v0[i] ? xs[col0 + e] : 0.0f;
                    xr[i][8 + e] = v1[i] ? xs[col0 + 256 + e] : 0.0f;
                }
            } else if (j < csubs) {
                const float *xc = xs + (j % slots) * kSubElems + lane * 8;
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    xr[i][e] = xc[e];
                    xr[i][8 + e] = xc[256 + e];
                }
            }
        }
    }

    if (producer) {
        if (lane == 0 && ok) {
            uint32_t s = primed % static_cast<uint32_t>(stages);
            uint32_t phase = primed == static_cast<uint32_t>(stages) ? 0u : 1u;  // parity to wait for
            for (uint32_t k = primed; k < total; ++k) {
                if (!mbar_wait(&empty_bar[s], phase)) {
                    *reinterpret_cast<volatile int *>(&abort_flag) = 1;
                    if (p.error) atomicExch(p.error, 2u);
                    break;
                }
                issue(k, s);
                issued = k + 1;
                if (++s == static_cast<uint32_t>(stages)) {
                    s = 0;
                    phase ^= 1u;
                }
            }
        }
    } else if (ok) {
        uint32_t s = 0, phase = 0;
        for (uint32_t k = 0; k < total; ++k) {
            if (!mbar_wait(&full_bar[s], phase)) {
                *reinterpret_cast<volatile int *>(&abort_flag) = 1;
                if (p.error && lane == 0) atomicExch(p.error, 2u);
                break;
            }
            const uint32_t m = (kPair == 2 && k >= cpr) ? 1u : 0u;
            const uint32_t sub0 = (k - m * cpr) * csubs;
            const uint32_t left = subs_per_range - sub0;
            const uint32_t nsub = left < csubs ? left : csubs;
            const uint4 *stage = reinterpret_cast<const uint4 *>(ring + static_cast<size_t>(s) * chunk_bytes);
#pragma unroll
            for (int i = 0; i < SETS; ++i) {
                const uint32_t j = static_cast<uint32_t>(warp) + 16u * i;
                if (j < nsub) {
                    const uint32_t g = sub0 + j;
                    const uint32_t row = g / slots, slot = g - row * slots;
                    uint4 w0, w1;
                    if constexpr (PART) {
                        const uint4 z = make_uint4(0, 0, 0, 0);
                        w0 = v0[i] ? stage[soff[i]] : z;
                        w1 = v1[i] ? stage[soff[i] + 32] : z;
                    } else {
                        w0 = stage[j * 64 + lane];
                        w1 = stage[j * 64 + 32 + lane];
                    }
                    const float a = dot8r(w0, xr[i], 0.0f);
                    const float b = dot8r(w1, xr[i] + 8, 0.0f);
                    const float sum = warp_sum(a + b);
                    if (lane == 0) partial[(row * slots + slot) * kPair + m] = sum;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty_bar[s]);
            if (*reinterpret_cast<volatile int *>(&abort_flag)) break;
            if (++s == static_cast<uint32_t>(stages)) {
                s = 0;
                phase ^= 1u;
            }
        }
    }
    __syncthreads();
    if (!ok || abort_flag) {
        // Drain: every copy that was issued lands before the CTA exits
        // (bounded waits; phases already complete return at once).
        if (producer && lane == 0)
            for (uint32_t k = issued > static_cast<uint32_t>(stages) ? issued - stages : 0; k < issued; ++k)
                mbar_wait(&full_bar[k % stages], (k / stages) & 1u);
        return;
    }
    if (p.trace && threadIdx.x == 0) {
        const uint64_t t = global_ns();
        trace_stamp(p.trace, 2, t);
        trace_stamp(p.trace, 3, t);
    }
    gemv_epilogue<EPI>(p, partial, u0, u1, slots, red);
}

// Bulk path applies when rows split into 512-column slots and a chunk (one
// row at most 64 slots) fits the ring.
inline bool gemv_bulk_shape(uint64_t cols) {
    return cols % 8 == 0 && bulk_slots(cols) <= 16ull * kMaxSets;
}
// Register sets a warp needs: one per 16 sub-ranges of a chunk.
inline int gemv_bulk_sets(uint64_t cols) {
    const uint32_t subs = bulk_chunk_subs(bulk_slots(cols));
    return subs <= 16 ? 1 : (subs <= 32 ? 2 : 4);
}
inline uint32_t gemv_bulk_chunk_bytes(uint64_t cols) {
    const uint32_t slots = bulk_slots(cols);
    return bulk_chunk_subs(slots) / slots * static_cast<uint32_t>(cols) * 2;
}
inline size_t gemv_bulk_smem(uint64_t cols, uint64_t rows_per_block, int pair, int stages) {
    return static_cast<size_t>(stages) * gemv_bulk_chunk_bytes(cols) +
           (((cols + 3) & ~3ull) + rows_per_block * bulk_slots(cols) * pair) * sizeof(float);
}

// Merge per-block argmax candidates: first maximal index, NaN -> UINT32_MAX
// (reference src/token.s:35-63). Writes the winner to *out and, when given,
// to the next decode step's token slot.
// With val2 (the blocks' runner-up values), margin receives best minus the
// largest value at any other index (the draft proposer's confidence).
__global__ void argmax_merge_kernel(const float *val, const uint32_t *idx, const uint32_t *nan_flag,
                                    uint32_t blocks, uint32_t *out, uint32_t *next_token, float *out_val,
                                    const float *val2, float *margin) {
    __shared__ float wv[32], ws[32];
    __shared__ uint32_t wi[32];
    __shared__ uint32_t wn[32];
    pdl_wait();
    const float ninf = -__int_as_float(0x7f800000);
    float bv = ninf, sv = ninf;
    uint32_t bi = 0xffffffffu, nan_seen = 0;
    for (uint32_t b = threadIdx.x; b < blocks; b += blockDim.x) {
        nan_seen |= nan_flag[b];
        top2_merge(val[b], idx[b], val2 ? val2[b] : ninf, bv, bi, sv);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        const float os = __shfl_xor_sync(0xffffffffu, sv, o);
        nan_seen |= __shfl_xor_sync(0xffffffffu, nan_seen, o);
        top2_merge(ov, oi, os, bv, bi, sv);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) {
        wv[warp] = bv;
        wi[warp] = bi;
        ws[warp] = sv;
        wn[warp] = nan_seen;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) {
            nan_seen |= wn[w];
            top2_merge(wv[w], wi[w], ws[w], bv, bi, sv);
        }
        const uint32_t result = nan_seen ? 0xffffffffu : bi;
        *out = result;
        if (next_token) *next_token = result;
        if (out_val) *out_val = bv;
        if (margin) *margin = __fsub_rn(bv, sv);
    }
}

// Greedy choice of every row of a [rows][n] logits block, two passes: grid
// (chunks, rows) of per-chunk candidates, then one merge block per row.
__global__ void rows_argmax_partial_kernel(const float *logits, uint64_t n, float *val, uint32_t *idx,
                                           uint32_t *nan_flag) {
    __shared__ float sv[32];
    __shared__ uint32_t si[32];
    __shared__ uint32_t sn[32];
    pdl_wait();
    const uint32_t row = blockIdx.y, chunk = blockIdx.x, chunks = gridDim.x;
    const uint64_t c0 = n * chunk / chunks, c1 = n * (chunk + 1) / chunks;
    const float *x = logits + row * n;
    float bv = -__int_as_float(0x7f800000);
    uint32_t bi = 0xffffffffu, nan_seen = 0;
    for (uint64_t i = c0 + threadIdx.x; i < c1; i += blockDim.x) {
        const float v = x[i];
        if (v != v) nan_seen = 1;
        else if (arg_better(v, static_cast<uint32_t>(i), bv, bi)) {
            bv = v;
            bi = static_cast<uint32_t>(i);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        nan_seen |= __shfl_xor_sync(0xffffffffu, nan_seen, o);
        if (arg_better(ov, oi, bv, bi)) {
            bv = ov;
            bi = oi;
        }
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) {
        sv[warp] = bv;
        si[warp] = bi;
        sn[warp] = nan_seen;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) {
            nan_seen |= sn[w];
            if (arg_better(sv[w], si[w], bv, bi)) {
                bv = sv[w];
                bi = si[w];
            }
        }
        val[row * chunks + chunk] = bv;
        idx[row * chunks + chunk] = bi;
        nan_flag[row * chunks + chunk] = nan_seen;
    }
    pdl_launch_dependents();
}

// One block per row: merge that row's chunk candidates (argmax_merge_kernel's
// rule) into out[row] (UINT32_MAX on NaN) and, when given, out_val[row].
__global__ void rows_argmax_merge_kernel(const float *val, const uint32_t *idx, const uint32_t *nan_flag,
                                         uint32_t chunks, uint32_t *out, float *out_val) {
    pdl_wait();
    if (threadIdx.x != 0) return;
    const uint32_t row = blockIdx.x;
    float bv = -__int_as_float(0x7f800000);
    uint32_t bi = 0xffffffffu, nan_seen = 0;
    for (uint32_t c = 0; c < chunks; ++c) {
        const uint32_t k = row * chunks + c;
        nan_seen |= nan_flag[k];
        if (arg_better(val[k], idx[k], bv, bi)) {
            bv = val[k];
            bi = idx[k];
        }
    }
    out[row] = nan_seen ? 0xffffffffu : bi;
    if (out_val) out_val[row] = bv;
}

}  // namespace plamo
