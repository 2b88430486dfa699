// Row-wise kernels of the layer-major prompt path (reference src/batch.s,
// src/prefill.s): embeddings, RMSNorm rows with fused residuals, SwiGLU rows,
// and the FP32-SIMT BF16 projection used for small token counts.
#pragma once
#include "common.cuh"
#include "../../include/plamo_synthetic.h"

namespace plamo {

// states[t] = FP32(embedding[ids[t]]) (reference src/token.s:6-33).
__global__ void embed_rows_kernel(const uint16_t *table, const uint32_t *ids, uint64_t vocab,
                                  uint64_t hidden, float *states, uint32_t *error) {
    pdl_wait();
    const uint32_t id = ids[blockIdx.x];
    if (id >= vocab) {
        if (threadIdx.x == 0) *error = 1;
        return;
    }
    const uint16_t *row = table + static_cast<uint64_t>(id) * hidden;
    float *out = states + static_cast<uint64_t>(blockIdx.x) * hidden;
    for (uint64_t i = threadIdx.x; i < hidden; i += blockDim.x) out[i] = bf16_to_f32(row[i]);
}

enum RowMode { ROW_NORM = 0, ROW_RESID = 1, ROW_RESID_NORM = 2 };

// FP32 -> BF16 terms hi = bf16(x), mid = bf16(x - hi), lo = bf16(x - hi - mid)
// (round to nearest even): the tcgen05 projections' view of an activation.
__device__ __forceinline__ void split3(float v, uint16_t *h, uint16_t *m, uint16_t *l) {
    const uint16_t a = plamo_bf16_round(v);
    const float r1 = __fsub_rn(v, __uint_as_float(static_cast<uint32_t>(a) << 16));
    const uint16_t b = plamo_bf16_round(r1);
    const float r2 = __fsub_rn(r1, __uint_as_float(static_cast<uint32_t>(b) << 16));
    *h = a;
    *m = b;
    *l = plamo_bf16_round(r2);
}

// Work the row kernels take over from their neighbours in the prompt and
// batch paths (zero-initialised: none):
//   split  - also write the BF16 terms of the kernel's output for the next
//            tcgen05 projection ([3][rows][width] planes), so no separate
//            split pass is needed;
//   bparts - the branch input arrives as `bsplits` split-K partial planes of
//            the previous projection ([bsplits][rows][width], plane bplane),
//            summed here in plane order instead of by a separate pass.
struct RowFuse {
    uint16_t *split;
    const float *bparts;
    uint32_t bsplits;
    uint64_t bplane;
};

__device__ __forceinline__ float4 fuse_branch4(const RowFuse &f, const float *b, uint64_t off) {
    if (f.bsplits <= 1) return ld4(b + off);
    float4 s = ld4(f.bparts + off);
    for (uint32_t z = 1; z < f.bsplits; ++z) {
        const float4 v = ld4(f.bparts + z * f.bplane + off);
        s = make_float4(__fadd_rn(s.x, v.x), __fadd_rn(s.y, v.y), __fadd_rn(s.z, v.z), __fadd_rn(s.w, v.w));
    }
    return s;
}
__device__ __forceinline__ float fuse_branch1(const RowFuse &f, const float *b, uint64_t off) {
    if (f.bsplits <= 1) return b[off];
    float s = f.bparts[off];
    for (uint32_t z = 1; z < f.bsplits; ++z) s = __fadd_rn(s, f.bparts[z * f.bplane + off]);
    return s;
}
__device__ __forceinline__ void fuse_split4(const RowFuse &f, uint64_t plane, uint64_t off, float4 v) {
    if (!f.split) return;
    uint16_t h[4], m[4], l[4];
    split3(v.x, &h[0], &m[0], &l[0]);
    split3(v.y, &h[1], &m[1], &l[1]);
    split3(v.z, &h[2], &m[2], &l[2]);
    split3(v.w, &h[3], &m[3], &l[3]);
    *reinterpret_cast<uint2 *>(f.split + off) = make_uint2(h[0] | (uint32_t(h[1]) << 16), h[2] | (uint32_t(h[3]) << 16));
    *reinterpret_cast<uint2 *>(f.split + plane + off) =
        make_uint2(m[0] | (uint32_t(m[1]) << 16), m[2] | (uint32_t(m[3]) << 16));
    *reinterpret_cast<uint2 *>(f.split + 2 * plane + off) =
        make_uint2(l[0] | (uint32_t(l[1]) << 16), l[2] | (uint32_t(l[3]) << 16));
}
__device__ __forceinline__ void fuse_split1(const RowFuse &f, uint64_t plane, uint64_t off, float v) {
    if (!f.split) return;
    split3(v, f.split + off, f.split + plane + off, f.split + 2 * plane + off);
}

// One CTA per token row:
//   ROW_NORM:       out = rmsnorm(states, w2, off2)
//   ROW_RESID:      states += rmsnorm(branch, w1, off1)
//   ROW_RESID_NORM: both, the norm reading the updated state.
// Rows of a multiple of 4 floats take 128-bit loads, each thread holding its
// float4s in registers between the two norms (up to 4 per thread).
template <int MODE>
__global__ void norm_rows_kernel(float *states, const float *branch, const uint16_t *w1, float off1,
                                 const uint16_t *w2, float off2, float *out, uint64_t hidden, RowFuse fuse) {
    __shared__ float red[32];
    pdl_wait();
    float *x = states + static_cast<uint64_t>(blockIdx.x) * hidden;
    const uint64_t row0 = static_cast<uint64_t>(blockIdx.x) * hidden;
    const uint64_t plane = static_cast<uint64_t>(gridDim.x) * hidden;
    const uint32_t nt = blockDim.x;
    if (hidden % 4 == 0 && hidden <= 16ull * nt) {
        const uint32_t n4 = static_cast<uint32_t>(hidden / 4);
        float4 st[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t i = threadIdx.x + k * nt;
            if (i < n4) st[k] = ld4(x + 4 * i);
        }
        if (MODE != ROW_NORM) {
            float4 br[4];
            uint2 wv[4];
            float s = 0.0f;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint32_t i = threadIdx.x + k * nt;
                if (i < n4) {
                    br[k] = fuse_branch4(fuse, branch, row0 + 4 * i);
                    wv[k] = *reinterpret_cast<const uint2 *>(w1 + 4 * i);
                    s += sq4(br[k]);
                }
            }
            const float inv = rms_inverse(block_sum(s, red), hidden);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint32_t i = threadIdx.x + k * nt;
                if (i < n4) {
                    const float4 v = apply4(br[k], inv, norm4(wv[k], off1));
                    st[k] = make_float4(__fadd_rn(st[k].x, v.x), __fadd_rn(st[k].y, v.y), __fadd_rn(st[k].z, v.z),
                                        __fadd_rn(st[k].w, v.w));
                    *reinterpret_cast<float4 *>(x + 4 * i) = st[k];
                }
            }
        }
        if (MODE != ROW_RESID) {
            float s = 0.0f;
            uint2 wv[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint32_t i = threadIdx.x + k * nt;
                if (i < n4) {
                    wv[k] = *reinterpret_cast<const uint2 *>(w2 + 4 * i);
                    s += sq4(st[k]);
                }
            }
            const float inv = rms_inverse(block_sum(s, red), hidden);
            float *o = out + static_cast<uint64_t>(blockIdx.x) * hidden;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint32_t i = threadIdx.x + k * nt;
                if (i < n4) {
                    const float4 v = apply4(st[k], inv, norm4(wv[k], off2));
                    *reinterpret_cast<float4 *>(o + 4 * i) = v;
                    fuse_split4(fuse, plane, row0 + 4 * i, v);
                }
            }
        }
        pdl_launch_dependents();
        return;
    }
    if (MODE != ROW_NORM) {
        float s = 0.0f;
        for (uint64_t i = threadIdx.x; i < hidden; i += blockDim.x) {
            const float b = fuse_branch1(fuse, branch, row0 + i);
            s += b * b;
        }
        const float inv = rms_inverse(block_sum(s, red), hidden);
        for (uint64_t i = threadIdx.x; i < hidden; i += blockDim.x)
            x[i] = __fadd_rn(x[i], rms_apply(fuse_branch1(fuse, branch, row0 + i), inv, w1[i], off1));
        __syncthreads();
    }
    if (MODE != ROW_RESID) {
        float s = 0.0f;
        for (uint64_t i = threadIdx.x; i < hidden; i += blockDim.x) s += x[i] * x[i];
        const float inv = rms_inverse(block_sum(s, red), hidden);
        float *o = out + static_cast<uint64_t>(blockIdx.x) * hidden;
        for (uint64_t i = threadIdx.x; i < hidden; i += blockDim.x) {
            o[i] = rms_apply(x[i], inv, w2[i], off2);
            fuse_split1(fuse, plane, row0 + i, o[i]);
        }
    }
    pdl_launch_dependents();
}

// In place: gu[t][i] = swiglu(gu[t][i], gu[t][I + i]) (reference src/batch.s:22-45).
// fuse.split: also the BF16 terms of the result, [3][tokens][inter].
// Grid (inter / 1024 rounded up, tokens), 256 threads: four consecutive
// units per thread (inter % 4 == 0), 128-bit loads and stores, no division.
__global__ void swiglu_rows4_kernel(float *gu, uint64_t inter, uint64_t tokens, RowFuse fuse) {
    pdl_wait();
    const uint64_t t = blockIdx.y, i = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
    if (i < inter) {
        float *row = gu + t * 2 * inter;
        const float4 g = ld4(row + i), u = ld4(row + inter + i);
        const float4 v = make_float4(swiglu(g.x, u.x), swiglu(g.y, u.y), swiglu(g.z, u.z), swiglu(g.w, u.w));
        *reinterpret_cast<float4 *>(row + i) = v;
        fuse_split4(fuse, inter * tokens, t * inter + i, v);
    }
    pdl_launch_dependents();
}

__global__ void swiglu_rows_kernel(float *gu, uint64_t inter, uint64_t tokens, RowFuse fuse) {
    pdl_wait();
    const uint64_t total = inter * tokens;
    for (uint64_t k = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; k < total;
         k += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint64_t t = k / inter, i = k % inter;
        float *row = gu + t * 2 * inter;
        const float v = swiglu(row[i], row[inter + i]);
        row[i] = v;
        fuse_split1(fuse, total, k, v);
    }
    pdl_launch_dependents();
}

// Y[t][r] = sum_k X[t][k] * W[r][k]: FP32 CUDA-core tiles of 64 tokens x 64
// rows x 32 columns, BF16 weights widened on load. Used for verification
// blocks and prompts; any shape and stride.
constexpr int kGemmBM = 64, kGemmBN = 64, kGemmBK = 32;
__global__ void __launch_bounds__(256) gemm_simt_kernel(const float *X, uint64_t xs, const uint16_t *W,
                                                        float *Y, uint64_t ys, uint64_t T, uint64_t R,
                                                        uint64_t K) {
    __shared__ float As[kGemmBK][kGemmBM + 4];
    __shared__ float Bs[kGemmBK][kGemmBN + 4];
    pdl_wait();
    const uint64_t t0 = static_cast<uint64_t>(blockIdx.y) * kGemmBM;
    const uint64_t r0 = static_cast<uint64_t>(blockIdx.x) * kGemmBN;
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    float acc[4][4] = {};
    for (uint64_t k0 = 0; k0 < K; k0 += kGemmBK) {
        for (int i = threadIdx.x; i < kGemmBM * kGemmBK; i += 256) {
            const int m = i / kGemmBK, k = i % kGemmBK;
            const uint64_t gt = t0 + m, gk = k0 + k;
            As[k][m] = (gt < T && gk < K) ? X[gt * xs + gk] : 0.0f;
            const uint64_t gr = r0 + m;
            Bs[k][m] = (gr < R && gk < K) ? bf16_to_f32(W[gr * K + gk]) : 0.0f;
        }
        __syncthreads();
#pragma unroll 8
        for (int k = 0; k < kGemmBK; ++k) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[k][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = Bs[k][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint64_t gt = t0 + ty * 4 + i;
        if (gt >= T) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint64_t gr = r0 + tx * 4 + j;
            if (gr < R) Y[gt * ys + gr] = acc[i][j];
        }
    }
    pdl_launch_dependents();
}

__global__ void fill_synthetic_bf16_kernel(uint16_t *dst, uint64_t count, uint64_t seed, float mean,
                                           float std) {
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x)
        dst[i] = plamo_synthetic_bf16(seed, i, mean, std);
}

// Rows [row0, row0+rows) x columns [col0, col0+cols) of the synthetic
// [*, full_cols] tensor `seed`, packed as [rows][cols].
__global__ void fill_synthetic_rows_kernel(uint16_t *dst, uint64_t rows, uint64_t cols, uint64_t seed, uint64_t row0,
                                           uint64_t col0, uint64_t full_cols, float mean, float std) {
    const uint64_t count = rows * cols;
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint64_t r = i / cols, col = i - r * cols;
        dst[i] = plamo_synthetic_bf16(seed, (row0 + r) * full_cols + col0 + col, mean, std);
    }
}

__global__ void fill_synthetic_f32_kernel(float *dst, uint64_t count, uint64_t seed, float mean,
                                          float std) {
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x)
        dst[i] = plamo_synthetic_f32(seed, i, mean, std);
}

// Read every byte once (warm-up of resident weights).
__global__ void touch_kernel(const uint4 *p, uint64_t n, uint32_t *sink) {
    uint32_t x = 0;
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint4 v = p[i];
        x ^= v.x ^ v.y ^ v.z ^ v.w;
    }
    if (x == 0x9e3779b9u) *sink = x;
}

}  // namespace plamo
