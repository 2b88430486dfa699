// Q/K head norm + RoPE, GQA attention over the KV ring, KV ring stores.
//
// KV layout in HBM (per layer): two FP32 rings K[ring][kh*dim] and
// V[ring][kh*dim] holding normalised, UNROTATED keys and values, exactly the
// rows the reference keeps in struct cache (reference src/cache.s). Logical
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
#include "common.cuh"

namespace plamo {

struct AttnLayer {
    const float *ring_k, *ring_v;  // [ring][kh*dim]
    float *ring_k_w, *ring_v_w;    // same, writable (stores)
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
};

// One CTA per (kv head, query token, key split). Keys of the split are
// staged in tiles of 32 rows, rotated at their local position, scored against
// the G = qh/kh query heads of the group, and folded into an online softmax
// whose exponentials are the reference's exp polynomial. The last CTA of a
// (token, kv head) merges the split partials in split order.
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(AttnParams p) {
    extern __shared__ __align__(16) float sm[];
    const uint64_t D = p.S.dim, half = D / 2, QH = p.S.qh, KH = p.S.kh, G = QH / KH;
    const uint64_t kh = blockIdx.x, t = blockIdx.y, split = blockIdx.z;
    const uint64_t KS = D + 1;          // padded key row: conflict-free column reads
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
    const uint64_t kvw = KH * D;

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
        for (uint64_t i = threadIdx.x; i < rows * half; i += blockDim.x) {
            const uint64_t r = i / half, d = i % half, key = base + r;
            const float *ksrc, *vsrc;
            if (key < P) {
                const uint64_t slot = key % p.L.ring;
                ksrc = p.L.ring_k + slot * kvw + kh * D;
                vsrc = p.L.ring_v + slot * kvw + kh * D;
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
        for (uint64_t i = threadIdx.x; i < G * rows; i += blockDim.x) {
            const uint64_t g = i / rows, r = i % rows;
            const float *qv = qs + g * D, *kv = kt + r * KS;
            float a = 0.0f;
            for (uint64_t d = 0; d < D; ++d) a = fmaf(qv[d], kv[d], a);
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
        for (uint64_t i = threadIdx.x; i < G * D; i += blockDim.x) {
            const uint64_t g = i / D, d = i % D;
            float a = __fmul_rn(acc[i], corr[g]);
            for (uint64_t r = 0; r < rows; ++r) a = fmaf(sc[g * kAttnTile + r], vt[r * D + d], a);
            acc[i] = a;
        }
        __syncthreads();
    }

    if (p.splits == 1) {
        for (uint64_t i = threadIdx.x; i < G * D; i += blockDim.x) {
            const uint64_t g = i / D, d = i % D;
            p.out[(t * QH + kh * G + g) * D + d] = __fdiv_rn(acc[i], lrow[g]);
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
        p.out[(t * QH + kh * G + g) * D + d] = __fdiv_rn(A, Ls);
    }
    __syncthreads();
    if (threadIdx.x == 0) p.tickets[t * KH + kh] = 0;
    pdl_launch_dependents();
}

inline size_t attention_smem_bytes(uint64_t G, uint64_t D) {
    return (G * D + kAttnTile * (D + 1) + kAttnTile * D + G * kAttnTile + G * D + 3 * G) *
           sizeof(float);
}

// Store the K/V rows of tokens [first, tokens) (normalised K, V from the QKV
// buffer) into ring slots (P + t) % ring. One CTA per token.
__global__ void kv_store_kernel(AttnLayer L, AttnShape S, const float *qkv, uint64_t first) {
    pdl_wait();
    const uint64_t t = first + blockIdx.x;
    const uint64_t P = *L.appended;
    const uint64_t kvw = S.kh * S.dim;
    const uint64_t slot = (P + t) % L.ring;
    const float *row = qkv + t * S.qkv_stride;
    for (uint64_t i = threadIdx.x; i < kvw; i += blockDim.x) {
        L.ring_k_w[slot * kvw + i] = row[S.qh * S.dim + i];
        L.ring_v_w[slot * kvw + i] = row[(S.qh + S.kh) * S.dim + i];
    }
    pdl_launch_dependents();
}

// Copy K/V rows of one candidate (kept per layer by a verification) to the
// ring slot of the next committed row.
__global__ void kv_commit_kernel(AttnLayer L, uint64_t kvw, const float *k_row, const float *v_row) {
    const uint64_t P = *L.appended;
    const uint64_t slot = P % L.ring;
    for (uint64_t i = threadIdx.x; i < kvw; i += blockDim.x) {
        L.ring_k_w[slot * kvw + i] = k_row[i];
        L.ring_v_w[slot * kvw + i] = v_row[i];
    }
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
    const uint64_t slot = (P - count + r) % L.ring;
    const uint64_t half = dim / 2;
    const float *c = L.table + r * dim, *s = c + half;
    for (uint64_t i = threadIdx.x; i < kvw; i += blockDim.x) {
        k_out[r * kvw + i] = L.ring_k[slot * kvw + i];
        v_out[r * kvw + i] = L.ring_v[slot * kvw + i];
    }
    for (uint64_t i = threadIdx.x; i < heads * half; i += blockDim.x) {
        const uint64_t h = i / half, d = i % half;
        const float a = L.ring_k[slot * kvw + h * dim + d], b = L.ring_k[slot * kvw + h * dim + d + half];
        rot_out[r * kvw + h * dim + d] = __fsub_rn(__fmul_rn(a, c[d]), __fmul_rn(b, s[d]));
        rot_out[r * kvw + h * dim + d + half] = __fadd_rn(__fmul_rn(b, c[d]), __fmul_rn(a, s[d]));
    }
}

// Upload view: token-major host rows [0, count) into ring slots 0..count-1
// (the request restarts with count committed rows).
__global__ void kv_scatter_kernel(float *ring_k, float *ring_v, uint64_t ring, uint64_t kvw,
                                  const float *k_in, const float *v_in) {
    const uint64_t r = blockIdx.x;
    const uint64_t slot = r % ring;
    for (uint64_t i = threadIdx.x; i < kvw; i += blockDim.x) {
        ring_k[slot * kvw + i] = k_in[r * kvw + i];
        ring_v[slot * kvw + i] = v_in[r * kvw + i];
    }
}

}  // namespace plamo
