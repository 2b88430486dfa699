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

namespace plamo {

enum GemvPrologue { PRO_X = 0, PRO_NORM = 1, PRO_RESID_NORM = 2, PRO_EMBED_NORM = 3 };
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
    uint32_t *arg_idx;            // ARGMAX: per-block best index
    uint32_t *arg_nan;            // ARGMAX: per-block NaN flag
    uint32_t *error;              // set to nonzero on an invalid token
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

// Build the FP32 input vector in shared memory. All blocks compute the same
// bits (same reduction shape), block 0 publishes state/normalised copies.
template <int PRO>
__device__ __forceinline__ bool gemv_prologue(const GemvParams &p, float *xs, float *red) {
    const uint64_t n = p.cols;
    const bool publish = blockIdx.x == 0;
    if (PRO == PRO_X) {
        for (uint64_t i = threadIdx.x; i < n; i += blockDim.x) xs[i] = p.x[i];
        return true;
    }
    if (PRO == PRO_EMBED_NORM) {
        const uint32_t token = *p.token;
        if (token >= p.vocab) {
            if (publish && threadIdx.x == 0) *p.error = 1;
            return false;
        }
        const uint16_t *row = p.embedding + static_cast<uint64_t>(token) * n;
        for (uint64_t i = threadIdx.x; i < n; i += blockDim.x) xs[i] = bf16_to_f32(row[i]);
    } else if (PRO == PRO_NORM) {
        for (uint64_t i = threadIdx.x; i < n; i += blockDim.x) xs[i] = p.state_in[i];
    } else {  // PRO_RESID_NORM: state + rmsnorm(branch, norm1, off1)
        float s = 0.0f;
        for (uint64_t i = threadIdx.x; i < n; i += blockDim.x) {
            const float b = p.branch[i];
            s += b * b;
        }
        const float inv = rms_inverse(block_sum(s, red), n);
        for (uint64_t i = threadIdx.x; i < n; i += blockDim.x)
            xs[i] = __fadd_rn(p.state_in[i], rms_apply(p.branch[i], inv, p.norm1[i], p.off1));
    }
    __syncthreads();
    float s = 0.0f;
    for (uint64_t i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = xs[i];
        s += v * v;
        if (publish && p.state_out) p.state_out[i] = v;
    }
    const float inv = rms_inverse(block_sum(s, red), n);
    for (uint64_t i = threadIdx.x; i < n; i += blockDim.x) {
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

// U: 256-column chunks per work item (U = 0: any shape, scalar loads).
template <int PRO, int EPI, int U>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(GemvParams p) {
    extern __shared__ __align__(16) float smem[];
    __shared__ float red[kGemvWarps];
    __shared__ float best_val[kGemvWarps];
    __shared__ uint32_t best_idx[kGemvWarps];
    __shared__ uint32_t any_nan;

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

    // Row pointer of work item j, pair member m.
    auto row_ptr = [&](uint64_t j, int m) -> const uint16_t * {
        const uint64_t unit = u0 + j / segs;
        const uint64_t row = m ? unit + half_rows : unit;
        return p.w + row * cols + (j % segs) * seg_cols;
    };

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

    pdl_wait();
    const bool ok = gemv_prologue<PRO>(p, xs, red);
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
            const float *xseg = xs + (j % segs) * seg_cols + lane * 8;
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
    pdl_launch_dependents();
    __syncthreads();

    // Fixed-order reduction of the segment partials, then the epilogue.
    float bv = -__int_as_float(0x7f800000);
    uint32_t bi = 0xffffffffu;
    bool saw_nan = false;
    for (uint64_t u = threadIdx.x; u < u1 - u0; u += blockDim.x) {
        float t0 = 0.0f, t1 = 0.0f;
        for (uint64_t s = 0; s < segs; ++s) {
            t0 += partial[(u * segs + s) * kPair];
            if (kPair == 2) t1 += partial[(u * segs + s) * kPair + 1];
        }
        const uint64_t unit = u0 + u;
        if (EPI == EPI_SWIGLU) {
            p.y[unit] = swiglu(t0, t1);
        } else {
            p.y[unit] = t0;
            if (EPI == EPI_ARGMAX) {
                if (t0 != t0) saw_nan = true;
                else if (arg_better(t0, static_cast<uint32_t>(unit), bv, bi)) {
                    bv = t0;
                    bi = static_cast<uint32_t>(unit);
                }
            }
        }
    }
    if (EPI == EPI_ARGMAX) {
        if (threadIdx.x == 0) any_nan = 0;
        __syncthreads();
        if (saw_nan) any_nan = 1;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (arg_better(ov, oi, bv, bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if (lane == 0) {
            best_val[warp] = bv;
            best_idx[warp] = bi;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            for (int w = 1; w < kGemvWarps; ++w)
                if (arg_better(best_val[w], best_idx[w], bv, bi)) {
                    bv = best_val[w];
                    bi = best_idx[w];
                }
            p.arg_val[blockIdx.x] = bv;
            p.arg_idx[blockIdx.x] = bi;
            p.arg_nan[blockIdx.x] = any_nan;
        }
    }
}

// Merge per-block argmax candidates: first maximal index, NaN -> UINT32_MAX
// (reference src/token.s:35-63). Writes the winner to *out and, when given,
// to the next decode step's token slot.
__global__ void argmax_merge_kernel(const float *val, const uint32_t *idx, const uint32_t *nan_flag,
                                    uint32_t blocks, uint32_t *out, uint32_t *next_token) {
    __shared__ float sv[32];
    __shared__ uint32_t si[32];
    __shared__ uint32_t sn[32];
    pdl_wait();
    float bv = -__int_as_float(0x7f800000);
    uint32_t bi = 0xffffffffu, nan_seen = 0;
    for (uint32_t b = threadIdx.x; b < blocks; b += blockDim.x) {
        nan_seen |= nan_flag[b];
        if (arg_better(val[b], idx[b], bv, bi)) {
            bv = val[b];
            bi = idx[b];
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
        const uint32_t result = nan_seen ? 0xffffffffu : bi;
        *out = result;
        if (next_token) *next_token = result;
    }
}

// Greedy choice of every row of a [rows][n] logits block (verification).
__global__ void rows_argmax_kernel(const float *logits, uint64_t n, uint32_t *out) {
    __shared__ float sv[32];
    __shared__ uint32_t si[32];
    __shared__ uint32_t sn[32];
    pdl_wait();
    const float *x = logits + blockIdx.x * n;
    float bv = -__int_as_float(0x7f800000);
    uint32_t bi = 0xffffffffu, nan_seen = 0;
    for (uint64_t i = threadIdx.x; i < n; i += blockDim.x) {
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
        out[blockIdx.x] = nan_seen ? 0xffffffffu : bi;
    }
}

}  // namespace plamo
