// One decode token in one launch (single GPU): every projection, the
// attention of every layer and the greedy choice of a PLaMo-3 decode step in
// one persistent kernel (reference runtime/metal_model.m:385-505 encodes the
// same step as one command buffer; src/forward.s:9-84 on the CPU).
//
// Why: a decode step streams every weight byte once (16.2 GB for the 8B
// profile) and is bound by HBM bandwidth. As a chain of kernels, each launch
// boundary drains the weight stream (the next projection's CTAs start only
// as SMs free up) and the latency-bound attention of each layer is exposed.
// Here one CTA per SM lives for the whole token:
//   * a producer warp streams this CTA's rows of EVERY projection of EVERY
//     layer, in step order, through one ring of 32 KB shared-memory stages
//     with cp.async.bulk (the TMA engine, 1-D copies, no tensor map, no
//     multicast) and full/empty mbarrier pairs. It never waits for a phase:
//     while the consumer warps wait at a grid barrier or run attention, the
//     ring fills with the next projection's rows, so the stream only pauses
//     when a pause is longer than the ring (about 3.5 us across the GPU);
//   * 16 consumer warps run the phases: the prologue that builds the
//     projection's input vector (embedding, residual add, RMSNorms, exactly
//     as the graph's projection prologues), the dot products of each staged
//     chunk (each warp keeps its slice of the input in registers), the
//     epilogue (store, SwiGLU, argmax candidates), then attention;
//   * phases are separated by grid barriers: one release add per CTA on a
//     monotonic 64-bit counter and an acquire poll, bounded by 2 s;
//   * attention of a layer is split over all CTAs (each KV head's rows in S
//     contiguous splits, one per CTA), each split writes its online-softmax
//     partials, and the last split of a head to arrive (an arrival counter)
//     merges them and writes the head group's output.
// Dot products are formed exactly as in gemv_bulk_kernel (per 512-column
// sub-range, the same lanes and order, slots summed in order), so the
// projections give the same bits as the graph's.
//
// Every wait is bounded (2 s of %globaltimer). On a timeout or an invalid
// token the CTA records an error code, stops issuing copies, drains the ones
// in flight and returns; the host resets the barrier counters after an error.
#pragma once
#include "attention.cuh"
#include "common.cuh"
#include "gemv.cuh"

namespace plamo {

// 16 consumer warps and one producer warp. A stage holds 16 sub-ranges of
// 512 columns (16 KB), one per consumer warp: a chunk is a whole number of
// rows when a row has at most 16 sub-ranges, else one part of a row of 32
// (two parts per row, the warp's column slot alternating between its two
// register sets with the chunk's parity).
constexpr int kPtConsumers = 16;
constexpr int kPtConsumerThreads = kPtConsumers * 32;
constexpr int kPtThreads = kPtConsumerThreads + 32;
constexpr uint32_t kPtStageSubs = kPtConsumers;
constexpr uint32_t kPtStageBytes = kPtStageSubs * kSubElems * 2;
constexpr int kPtMaxStages = 12;
constexpr int kPtDefaultStages = 6;  // 96 KB in flight per SM
constexpr uint32_t kPtMaxSlots = 2 * kPtStageSubs;  // rows of at most 16384 columns
constexpr uint32_t kPtTile = 16;                // attention key rows per tile
constexpr uint32_t kPtMaxG = 16;                // query heads per KV head
constexpr uint32_t kPtMaxSplits = 64;           // attention splits per KV head
constexpr uint32_t kPtMaxHidden = 4 * 4 * kPtConsumerThreads;  // 4 float4 per consumer thread
constexpr uint64_t kPtWaitNs = 2000000000ull;
constexpr float kPtPostMixer = 0.2f;                  // reference src/layer.s:51
constexpr float kPtPostMlp = 0.08944271909999159f;    // reference src/model.s:112

struct PtLayer {
    const uint16_t *qkv_w, *o_w, *gu, *down;
    const uint16_t *pre, *post, *mpre, *mpost;
    AttnLayer attn;
};

struct PtParams {
    const PtLayer *layers;  // [L] device records
    uint32_t L, H, QH, KH, AW, I, QW, head_rows;
    uint64_t vocab;
    const uint16_t *emb, *norm, *head;
    uint32_t *token;         // this step's token; receives the greedy choice
    uint32_t *next;          // [0] greedy choice, [1] error code, [2] top-2 margin bits
    float *state[2];         // hidden state ping-pong (as the graph uses it)
    float *normalized, *logits, *qkv, *attn, *branch, *mid;
    float *apart;            // attention partials [KH][S][G * (128 + 2)]
    uint32_t *head_arrive;   // [KH] arrival counters of the attention splits
    unsigned long long *bar; // grid barrier counter (monotonic)
    unsigned long long *gen; // completed launches (barrier targets derive from it)
    float *arg_val, *arg_val2;
    uint32_t *arg_idx, *arg_nan;  // [grid] head candidates
    uint64_t *appended;      // [L] committed rows, +1 at the end of the step
    uint32_t S;              // attention splits per KV head
    uint32_t stages;
    uint32_t piece;          // bytes per bulk copy (a stage is filled by several)
    // Optional (null: off) %globaltimer stamps of block 0: [0] start, then
    // [1 + b] when its consumers passed grid barrier b (B = 5L + 1 of them),
    // then [1 + B + ph] when its producer issued the first chunk of
    // projection ph (4L + 1 of them).
    unsigned long long *trace;
};

// Phase geometry of projection `ph` (4 per layer: qkv, o, gate_up, down;
// then the head) for this CTA. parts = 1: a chunk is rpc whole rows; parts =
// 2: a chunk is half a row (rpc = 1, cpr counts half rows).
struct PtGemv {
    const uint16_t *w;
    uint32_t units, cols, pair;
    uint32_t slots, parts, rpc, u0, n, cpr;
};

__device__ __forceinline__ PtGemv pt_gemv(const PtParams &p, uint32_t ph) {
    PtGemv g;
    if (ph == 4 * p.L) {
        g.w = p.head, g.units = p.head_rows, g.cols = p.H, g.pair = 1;
    } else {
        const PtLayer &L = p.layers[ph >> 2];
        switch (ph & 3) {
        case 0: g.w = L.qkv_w, g.units = p.QW, g.cols = p.H, g.pair = 1; break;
        case 1: g.w = L.o_w, g.units = p.H, g.cols = p.AW, g.pair = 1; break;
        case 2: g.w = L.gu, g.units = p.I, g.cols = p.H, g.pair = 2; break;
        default: g.w = L.down, g.units = p.H, g.cols = p.I, g.pair = 1; break;
        }
    }
    g.slots = g.cols / kSubElems;
    g.parts = g.slots > kPtStageSubs ? 2u : 1u;
    g.rpc = g.parts == 1 ? kPtStageSubs / g.slots : 1u;
    g.u0 = static_cast<uint32_t>(static_cast<uint64_t>(g.units) * blockIdx.x / gridDim.x);
    g.n = static_cast<uint32_t>(static_cast<uint64_t>(g.units) * (blockIdx.x + 1) / gridDim.x) - g.u0;
    g.cpr = g.parts == 1 ? (g.n + g.rpc - 1) / g.rpc : 2 * g.n;
    return g;
}

__device__ __forceinline__ void pt_consumer_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kPtConsumerThreads) : "memory");
}
// Consumer barrier that also returns, to every consumer thread, whether any
// of them passed `v` true: every decision that skips a later barrier is made
// from this value, so all 16 warps always take the same path (a named
// barrier that some warp never reaches would never complete).
__device__ __forceinline__ bool pt_sync_any(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 q, %1, 0;\n\t"
        "bar.red.or.pred p, 1, %2, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(v)), "n"(kPtConsumerThreads)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ unsigned long long ld_acquire_gpu_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_gpu_add(unsigned long long *p, unsigned long long v) {
    asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ bool pt_failed(const PtParams &p) {
    return *reinterpret_cast<const volatile uint32_t *>(p.next + 1) != 0u;
}
__device__ __forceinline__ void pt_fail(const PtParams &p, uint32_t code, volatile int *abort_flag) {
    atomicCAS(p.next + 1, 0u, code);
    *abort_flag = 1;
}

// Deterministic sum over the 512 consumer threads (fixed order).
__device__ __forceinline__ float pt_sum(float v, float *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    pt_consumer_sync();
    if (lane == 0) red[warp] = v;
    pt_consumer_sync();
    float total = 0.0f;
#pragma unroll
    for (int i = 0; i < kPtConsumers; ++i) total += red[i];
    return total;
}

// Grid barrier `b` of this launch (consumers): every consumer's global
// writes of the phase are ordered before this CTA's arrival; the poll ends
// once every CTA has arrived. False on a timeout or another CTA's failure.
__device__ __forceinline__ bool pt_grid_sync(const PtParams &p, unsigned long long gen, uint32_t b, uint32_t B,
                                             volatile int *abort_flag) {
    pt_consumer_sync();
    if (threadIdx.x == 0 && !*abort_flag) {
        const unsigned long long target = (gen * B + b + 1) * gridDim.x;
        __threadfence();
        red_release_gpu_add(p.bar, 1ull);
        uint64_t start = 0;
        while (ld_acquire_gpu_u64(p.bar) < target) {
            if (pt_failed(p)) {
                *abort_flag = 1;
                break;
            }
            if (!start) start = global_ns();
            else if (global_ns() - start > kPtWaitNs) {
                pt_fail(p, 5u, abort_flag);
                break;
            }
        }
        __threadfence();
        if (p.trace && blockIdx.x == 0) p.trace[1 + b] = global_ns();
    }
    return !pt_sync_any(*abort_flag);
}

// Input vector of a normalised projection: xs = rmsnorm(state_in [+ rmsnorm(branch)], norm2).
// PRO_EMBED_NORM when `token` is given; block 0 publishes the state (and the
// normalised vector when norm_out is set). Same arithmetic as gemv_prologue.
__device__ __noinline__ bool pt_norm_input(const PtParams &p, uint32_t token, bool embed, const float *state_in,
                                              const float *branch, const uint16_t *norm1, float off1,
                                              const uint16_t *norm2, float off2, float *state_out, float *norm_out,
                                              float *xs, float *red) {
    const uint32_t n4 = p.H / 4, nt = kPtConsumerThreads;
    const bool publish = blockIdx.x == 0;
    float4 st[4], br[4];
    uint2 w1[4], w2[4];
    const uint16_t *erow = p.emb + static_cast<uint64_t>(token) * p.H;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint32_t i = threadIdx.x + k * nt;
        if (i < n4) {
            if (embed) {
                const uint2 e = *reinterpret_cast<const uint2 *>(erow + 4 * i);
                st[k] = make_float4(bf16_lo(e.x), bf16_hi(e.x), bf16_lo(e.y), bf16_hi(e.y));
            } else {
                st[k] = __ldcg(reinterpret_cast<const float4 *>(state_in) + i);
                br[k] = __ldcg(reinterpret_cast<const float4 *>(branch) + i);
                w1[k] = *reinterpret_cast<const uint2 *>(norm1 + 4 * i);
            }
            w2[k] = *reinterpret_cast<const uint2 *>(norm2 + 4 * i);
        }
    }
    if (!embed) {
        float s = 0.0f;
#pragma unroll
        for (int k = 0; k < 4; ++k)
            if (threadIdx.x + k * nt < n4) s += sq4(br[k]);
        const float inv = rms_inverse(pt_sum(s, red), p.H);
#pragma unroll
        for (int k = 0; k < 4; ++k)
            if (threadIdx.x + k * nt < n4) {
                const float4 b = apply4(br[k], inv, norm4(w1[k], off1));
                st[k] = make_float4(__fadd_rn(st[k].x, b.x), __fadd_rn(st[k].y, b.y), __fadd_rn(st[k].z, b.z),
                                    __fadd_rn(st[k].w, b.w));
            }
    }
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint32_t i = threadIdx.x + k * nt;
        if (i < n4) {
            s += sq4(st[k]);
            if (publish) reinterpret_cast<float4 *>(state_out)[i] = st[k];
        }
    }
    const float inv = rms_inverse(pt_sum(s, red), p.H);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint32_t i = threadIdx.x + k * nt;
        if (i < n4) {
            const float4 v = apply4(st[k], inv, norm4(w2[k], off2));
            reinterpret_cast<float4 *>(xs)[i] = v;
            if (publish && norm_out) reinterpret_cast<float4 *>(norm_out)[i] = v;
        }
    }
    pt_consumer_sync();
    return true;
}

// Consumer side of one projection phase: register slices of the input
// (from shared `xs`, or from global `xg` written by other CTAs), the staged
// chunks in ring order, per-(row, slot) partials. Returns the ring position
// after the phase, or kPtAbort after an abort (the same value in every
// consumer thread). The epilogues below then reduce the partials.
constexpr uint32_t kPtAbort = 0xffffffffu;
__device__ __noinline__ uint32_t pt_stream(const PtParams &p, const PtGemv g, const float *xs, const float *xg,
                                           unsigned char *ring, uint64_t *full_bar, uint64_t *empty_bar,
                                           uint32_t chunk, float *partial, volatile int *abort_flag) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // This warp's column slots: warp % slots (whole-row chunks), or warp in
    // the first part of a row and warp + 16 in the second (which holds the
    // row's last slots - 16 sub-ranges).
    const uint32_t csubs = g.parts == 1 ? g.rpc * g.slots : kPtStageSubs;
    float xr[2][16];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const bool mine = g.parts == 1 ? (i == 0 && static_cast<uint32_t>(warp) < csubs)
                                       : warp + kPtStageSubs * i < g.slots;
        if (mine) {
            const uint32_t col = (g.parts == 1 ? warp % g.slots : warp + kPtStageSubs * i) * kSubElems + lane * 8;
            if (xg) {
                const float4 a = __ldcg(reinterpret_cast<const float4 *>(xg + col));
                const float4 b = __ldcg(reinterpret_cast<const float4 *>(xg + col + 4));
                const float4 c = __ldcg(reinterpret_cast<const float4 *>(xg + col + 256));
                const float4 d = __ldcg(reinterpret_cast<const float4 *>(xg + col + 260));
                xr[i][0] = a.x, xr[i][1] = a.y, xr[i][2] = a.z, xr[i][3] = a.w;
                xr[i][4] = b.x, xr[i][5] = b.y, xr[i][6] = b.z, xr[i][7] = b.w;
                xr[i][8] = c.x, xr[i][9] = c.y, xr[i][10] = c.z, xr[i][11] = c.w;
                xr[i][12] = d.x, xr[i][13] = d.y, xr[i][14] = d.z, xr[i][15] = d.w;
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    xr[i][e] = xs[col + e];
                    xr[i][8 + e] = xs[col + 256 + e];
                }
            }
        } else {
#pragma unroll
            for (int e = 0; e < 16; ++e) xr[i][e] = 0.0f;
        }
    }
    const uint32_t stages = p.stages;
    const uint32_t total = g.pair * g.cpr;
    const uint4 *ring4 = reinterpret_cast<const uint4 *>(ring);
    uint32_t s = chunk % stages, parity = (chunk / stages) & 1u;
    // After an abort the remaining chunks are skipped without waiting, so
    // every warp still reaches the barrier after the loop.
    for (uint32_t k = 0; k < total; ++k) {
        if (!*abort_flag) {
            // Every lane waits (each then sees the copied bytes); the warp acts
            // on the common result so its shuffles below stay convergent.
            if (!__all_sync(0xffffffffu, mbar_wait(&full_bar[s], parity))) {
                if (lane == 0) pt_fail(p, 2u, abort_flag);
            } else {
                const uint32_t m = k >= g.cpr ? 1u : 0u;
                const uint32_t kc = k - m * g.cpr;
                uint32_t row, slot, nsub;
                bool odd = false;
                if (g.parts == 1) {
                    const uint32_t rows = min(g.rpc, g.n - kc * g.rpc);
                    nsub = rows * g.slots;
                    const uint32_t r = static_cast<uint32_t>(warp) / g.slots;
                    row = kc * g.rpc + r;
                    slot = warp - r * g.slots;
                } else {
                    odd = kc & 1u;
                    nsub = odd ? g.slots - kPtStageSubs : kPtStageSubs;
                    row = kc >> 1;
                    slot = warp + (odd ? kPtStageSubs : 0u);
                }
                if (static_cast<uint32_t>(warp) < nsub) {
                    const uint4 *stage = ring4 + static_cast<size_t>(s) * (kPtStageBytes / 16);
                    const uint4 w0 = stage[warp * 64 + lane], w1 = stage[warp * 64 + 32 + lane];
                    float a, b;
                    if (odd) {
                        a = dot8r(w0, xr[1], 0.0f);
                        b = dot8r(w1, xr[1] + 8, 0.0f);
                    } else {
                        a = dot8r(w0, xr[0], 0.0f);
                        b = dot8r(w1, xr[0] + 8, 0.0f);
                    }
                    const float sum = warp_sum(a + b);
                    if (lane == 0) partial[(row * g.slots + slot) * g.pair + m] = sum;
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty_bar[s]);
            }
        }
        if (++s == stages) {
            s = 0;
            parity ^= 1u;
        }
    }
    return pt_sync_any(*abort_flag) ? kPtAbort : chunk + total;
}

// Epilogues: per-unit sums of the slots, in slot order.
__device__ __noinline__ void pt_store_epilogue(const PtGemv g, const float *partial, float *y) {
    for (uint32_t u = threadIdx.x; u < g.n; u += kPtConsumerThreads) {
        float t0 = 0.0f;
        for (uint32_t s = 0; s < g.slots; ++s) t0 += partial[u * g.slots + s];
        y[g.u0 + u] = t0;
    }
}
// SwiGLU of every gate/up unit pair of this CTA.
__device__ __noinline__ void pt_swiglu_epilogue(const PtGemv g, const float *partial, float *y) {
    for (uint32_t u = threadIdx.x; u < g.n; u += kPtConsumerThreads) {
        float t0 = 0.0f, t1 = 0.0f;
        for (uint32_t s = 0; s < g.slots; ++s) {
            t0 += partial[(u * g.slots + s) * 2];
            t1 += partial[(u * g.slots + s) * 2 + 1];
        }
        y[g.u0 + u] = swiglu(t0, t1);
    }
}
// Head: logits, and this CTA's greedy candidate (first maximum, runner-up
// value, NaN flag) for the merge at the end of the step.
__device__ __noinline__ void pt_head_epilogue(const PtParams &p, const PtGemv g, const float *partial, float *y) {
    __shared__ float cand_v[kPtConsumers], cand_s[kPtConsumers];
    __shared__ uint32_t cand_i[kPtConsumers], cand_n[kPtConsumers];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float bv = -__int_as_float(0x7f800000), sv = bv;
    uint32_t bi = 0xffffffffu;
    bool saw_nan = false;
    for (uint32_t u = threadIdx.x; u < g.n; u += kPtConsumerThreads) {
        float t0 = 0.0f;
        for (uint32_t s = 0; s < g.slots; ++s) t0 += partial[u * g.slots + s];
        const uint32_t unit = g.u0 + u;
        y[unit] = t0;
        if (t0 != t0) saw_nan = true;
        else top2_merge(t0, unit, -__int_as_float(0x7f800000), bv, bi, sv);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        const float os = __shfl_xor_sync(0xffffffffu, sv, o);
        top2_merge(ov, oi, os, bv, bi, sv);
    }
    const uint32_t any_nan = __any_sync(0xffffffffu, saw_nan);
    if (lane == 0) {
        cand_v[warp] = bv;
        cand_i[warp] = bi;
        cand_s[warp] = sv;
        cand_n[warp] = any_nan;
    }
    pt_consumer_sync();
    if (threadIdx.x == 0) {
        uint32_t nan_seen = cand_n[0];
        for (int w = 1; w < kPtConsumers; ++w) {
            top2_merge(cand_v[w], cand_i[w], cand_s[w], bv, bi, sv);
            nan_seen |= cand_n[w];
        }
        p.arg_val[blockIdx.x] = bv;
        p.arg_val2[blockIdx.x] = sv;
        p.arg_idx[blockIdx.x] = bi;
        p.arg_nan[blockIdx.x] = nan_seen;
    }
}

// Attention shared memory (floats) for G query heads per KV head and S splits.
__host__ __device__ inline uint32_t pt_attention_floats(uint32_t G, uint32_t S) {
    return G * 128                   // qs
           + kPtTile * kD128Stride   // kt (raw, then rotated in place)
           + kPtTile * 128           // tab
           + kPtTile * 128           // vt
           + G * kPtTile             // sc
           + G * 128                 // acc
           + 2 * 128                 // knew, vnew
           + 3 * G                   // m, l, corr
           + G * (S + 1);            // merge weights and denominators
}

// Attention of layer `l` for this CTA's (KV head, split), then the merge of
// the head's splits by the last split to finish (reference src/attention.s,
// src/qkv.s head norms, src/cache.s append, src/cache_rope.s local-position
// rotation; the same operations as decode_attention128_body).
__device__ __noinline__ void pt_attention(const PtParams &p, uint32_t l, float *sm) {
    constexpr uint32_t D = 128, HD = 64, KS = kD128Stride, T = kPtTile;
    const AttnLayer &A = p.layers[l].attn;
    const uint32_t G = p.QH / p.KH, S = p.S;
    const uint32_t item = blockIdx.x;
    if (item >= p.KH * S) return;
    const uint32_t kh = item / S, split = item - kh * S;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t nt = kPtConsumerThreads;
    float *qs = sm;
    float *kt = qs + G * D;
    float *tab = kt + T * KS;
    float *vt = tab + T * D;
    float *sc = vt + T * D;
    float *acc = sc + G * T;
    float *knew = acc + G * D;
    float *vnew = knew + D;
    float *mrow = vnew + D;
    float *lrow = mrow + G;
    float *corr = lrow + G;
    float *wmerge = corr + G;  // [G][S] then [G] denominators

    const uint64_t P = __ldcg(A.appended);
    const uint64_t lo = window_start(A, P, 0);
    const uint32_t n = static_cast<uint32_t>(P + 1 - lo);
    const uint64_t k0 = lo + static_cast<uint64_t>(n) * split / S;
    const uint64_t k1 = lo + static_cast<uint64_t>(n) * (split + 1) / S;

    auto stage = [&](uint64_t base, uint32_t rows) {
        for (uint32_t i = threadIdx.x; i < rows * 32; i += nt) {
            const uint32_t r = i >> 5, c = (i & 31) * 4;
            const uint64_t key = base + r;
            cp_async16(tab + r * D + c, A.table + (key - lo) * D + c);
            if (key < P) {
                cp_async16(kt + r * KS + c, kv_key(A, key) + kh * D + c);
                cp_async16(vt + r * D + c, kv_value(A, key) + kh * D + c);
            }
        }
        cp_async_commit();
    };
    if (k0 < k1) stage(k0, static_cast<uint32_t>(k1 - k0 < T ? k1 - k0 : T));

    // Query heads of the group (one warp each), normalised and rotated at the
    // query's local position n - 1.
    const float *table_q = A.table + static_cast<uint64_t>(n - 1) * D;
    for (uint32_t g = warp; g < G; g += kPtConsumers) {
        const float *x = p.qkv + static_cast<uint64_t>(kh * G + g) * D;
        float4 a = make_float4(0, 0, 0, 0), b = a, c = a, sn = a;
        uint2 wa = make_uint2(0, 0), wb = wa;
        if (lane < 16) {
            a = __ldcg(reinterpret_cast<const float4 *>(x + 4 * lane));
            b = __ldcg(reinterpret_cast<const float4 *>(x + HD + 4 * lane));
            wa = *reinterpret_cast<const uint2 *>(A.qn + 4 * lane);
            wb = *reinterpret_cast<const uint2 *>(A.qn + HD + 4 * lane);
            c = ld4(table_q + 4 * lane);
            sn = ld4(table_q + HD + 4 * lane);
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
            *reinterpret_cast<float4 *>(qs + g * D + HD + 4 * lane) = hi4;
        }
    }
    // The new row (normalised K, unrotated, and V): stored to the ring by the
    // split that ends at it; no split of this launch reads that slot.
    const bool has_new = k1 == P + 1;
    if (has_new && warp == kPtConsumers - 1) {
        const float *x = p.qkv + static_cast<uint64_t>(p.QH + kh) * D;
        const float *v = p.qkv + static_cast<uint64_t>(p.QH + p.KH + kh) * D;
        const float4 xk = __ldcg(reinterpret_cast<const float4 *>(x + 4 * lane));
        const float4 xv = __ldcg(reinterpret_cast<const float4 *>(v + 4 * lane));
        const uint2 wk = *reinterpret_cast<const uint2 *>(A.kn + 4 * lane);
        const float inv = rms_inverse(warp_sum(sq4(xk)), D);
        const float4 k4 = apply4(xk, inv, norm4(wk, 1.0f));
        *reinterpret_cast<float4 *>(knew + 4 * lane) = k4;
        *reinterpret_cast<float4 *>(vnew + 4 * lane) = xv;
        *reinterpret_cast<float4 *>(kv_key(A, P) + kh * D + 4 * lane) = k4;
        *reinterpret_cast<float4 *>(kv_value(A, P) + kh * D + 4 * lane) = xv;
    }
    for (uint32_t i = threadIdx.x; i < G * D; i += nt) acc[i] = 0.0f;
    for (uint32_t g = threadIdx.x; g < G; g += nt) {
        mrow[g] = -__int_as_float(0x7f800000);
        lrow[g] = 0.0f;
    }

    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(D)));
    for (uint64_t base = k0; base < k1; base += T) {
        const uint32_t rows = static_cast<uint32_t>(k1 - base < T ? k1 - base : T);
        cp_async_wait_all();
        pt_consumer_sync();
        if (base + rows == P + 1) {
            const uint32_t r = rows - 1;
            for (uint32_t i = threadIdx.x; i < D; i += nt) {
                kt[r * KS + i] = knew[i];
                vt[r * D + i] = vnew[i];
            }
            pt_consumer_sync();
        }
        for (uint32_t i = threadIdx.x; i < rows * 16; i += nt) {
            const uint32_t r = i >> 4, d = (i & 15) * 4;
            const float4 a = ld4(kt + r * KS + d), b = ld4(kt + r * KS + HD + d);
            const float4 c = ld4(tab + r * D + d), sn = ld4(tab + r * D + HD + d);
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
            *reinterpret_cast<float4 *>(kt + r * KS + HD + d) = hi4;
        }
        pt_consumer_sync();
        // Scores: one (head, key) per thread, sequential FMA over the head dim.
        for (uint32_t i = threadIdx.x; i < G * rows; i += nt) {
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
            sc[g * T + r] = __fmul_rn(a, scale);
        }
        pt_consumer_sync();
        // Online softmax per head (one warp each, lanes over the tile's keys).
        for (uint32_t g = warp; g < G; g += kPtConsumers) {
            const float ninf = -__int_as_float(0x7f800000);
            const float v0 = lane < static_cast<int>(rows) ? sc[g * T + lane] : ninf;
            const float m = fmaxf(mrow[g], warp_max(v0));
            const float e0 = lane < static_cast<int>(rows) ? plamo_exp(__fsub_rn(v0, m)) : 0.0f;
            if (lane < static_cast<int>(rows)) sc[g * T + lane] = e0;
            const float tile_sum = warp_sum(e0);
            if (lane == 0) {
                const float cr = plamo_exp(__fsub_rn(mrow[g], m));
                lrow[g] = __fadd_rn(__fmul_rn(lrow[g], cr), tile_sum);
                mrow[g] = m;
                corr[g] = cr;
            }
        }
        pt_consumer_sync();
        for (uint32_t i = threadIdx.x; i < G * 32; i += nt) {
            const uint32_t g = i >> 5, d = (i & 31) * 4;
            float4 a = ld4(acc + g * D + d);
            const float cr = corr[g];
            a = make_float4(__fmul_rn(a.x, cr), __fmul_rn(a.y, cr), __fmul_rn(a.z, cr), __fmul_rn(a.w, cr));
            const float *sg = sc + g * T;
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
        pt_consumer_sync();
        const uint64_t next = base + T;
        if (next < k1) stage(next, static_cast<uint32_t>(k1 - next < T ? k1 - next : T));
    }

    // This split's partials: acc [G][128], then m [G], l [G].
    const uint32_t pf = G * (D + 2);
    float *mine = p.apart + (static_cast<uint64_t>(kh) * S + split) * pf;
    for (uint32_t i = threadIdx.x; i < G * D; i += nt) mine[i] = acc[i];
    for (uint32_t g = threadIdx.x; g < G; g += nt) {
        mine[G * D + g] = mrow[g];
        mine[G * D + G + g] = lrow[g];
    }
    __shared__ uint32_t last;
    pt_consumer_sync();
    if (threadIdx.x == 0) {
        __threadfence();
        last = (atomicAdd(p.head_arrive + kh, 1u) + 1u) % S == 0u;
        __threadfence();
    }
    pt_consumer_sync();
    if (!last) return;

    // Merge of the head's S splits (fixed split order). Every split's (m, l)
    // is fetched at once into shared memory (one L2 round trip), then the
    // weights; the weighted sums keep kPtMergeBatch loads in flight.
    const float *parts = p.apart + static_cast<uint64_t>(kh) * S * pf;
    float *ms = kt;  // [S][G] split maxima, then [S][G] split sums (the key tile is free now)
    for (uint32_t i = threadIdx.x; i < S * G; i += nt) {
        const uint32_t r = i / G, g = i - r * G;
        ms[i] = __ldcg(parts + r * pf + G * D + g);
        ms[S * G + i] = __ldcg(parts + r * pf + G * D + G + g);
    }
    pt_consumer_sync();
    for (uint32_t g = threadIdx.x; g < G; g += nt) {
        float M = -__int_as_float(0x7f800000);
        for (uint32_t r = 0; r < S; ++r) M = fmaxf(M, ms[r * G + g]);
        float Ls = 0.0f;
        for (uint32_t r = 0; r < S; ++r) {
            const float e = plamo_exp(__fsub_rn(ms[r * G + g], M));
            wmerge[g * S + r] = e;
            Ls = fmaf(ms[S * G + r * G + g], e, Ls);
        }
        wmerge[G * S + g] = Ls;
    }
    pt_consumer_sync();
    constexpr uint32_t kPtMergeBatch = 16;
    for (uint32_t i = threadIdx.x; i < G * D; i += nt) {
        const uint32_t g = i / D;
        const float *w = wmerge + g * S;
        float a = 0.0f;
        for (uint32_t r0 = 0; r0 < S; r0 += kPtMergeBatch) {
            float v[kPtMergeBatch];
#pragma unroll
            for (uint32_t k = 0; k < kPtMergeBatch; ++k)
                v[k] = r0 + k < S ? __ldcg(parts + (r0 + k) * pf + i) : 0.0f;
#pragma unroll
            for (uint32_t k = 0; k < kPtMergeBatch; ++k)
                if (r0 + k < S) a = fmaf(v[k], w[r0 + k], a);
        }
        p.attn[static_cast<uint64_t>(kh * G) * D + i] = __fdiv_rn(a, wmerge[G * S + g]);
    }
}

// Parameters stay in the constant parameter space (__grid_constant__): the
// phase functions read them in place instead of from a per-thread copy.
__global__ void __launch_bounds__(kPtThreads, 1) decode_token_kernel(const __grid_constant__ PtParams p) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t full_bar[kPtMaxStages];
    __shared__ __align__(8) uint64_t empty_bar[kPtMaxStages];
    __shared__ float red[32];
    __shared__ int abort_flag_s;
    volatile int *abort_flag = &abort_flag_s;

    const uint32_t stages = p.stages;
    unsigned char *ring = smem_raw;
    float *work = reinterpret_cast<float *>(smem_raw + static_cast<size_t>(stages) * kPtStageBytes);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t phases = 4 * p.L + 1;
    const uint32_t B = 5 * p.L + 1;  // grid barriers per launch

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < stages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], kPtConsumers);
        }
        abort_flag_s = 0;
        fence_barrier_init();
    }
    __syncthreads();
    const unsigned long long gen = __ldcg(p.gen);
    if (p.trace && blockIdx.x == 0 && threadIdx.x == 0) p.trace[0] = global_ns();

    if (warp == kPtConsumers) {
        // Producer: every projection's rows of this CTA, in step order.
        if (lane != 0) return;
        const uint64_t policy = evict_first_policy();
        uint32_t issued = 0;
        bool stop = false;
        for (uint32_t ph = 0; ph < phases && !stop; ++ph) {
            const PtGemv g = pt_gemv(p, ph);
            const uint32_t total = g.pair * g.cpr;
            for (uint32_t k = 0; k < total; ++k) {
                const uint32_t s = issued % stages;
                if (issued >= stages) {
                    const uint32_t parity = ((issued / stages) - 1) & 1u;
                    bool ready = mbar_try_wait(&empty_bar[s], parity);
                    uint64_t start = 0;
                    while (!ready && !*abort_flag) {
                        if (!start) start = global_ns();
                        else if (global_ns() - start > kPtWaitNs) {
                            pt_fail(p, 2u, abort_flag);
                            break;
                        }
                        ready = mbar_try_wait(&empty_bar[s], parity);
                    }
                    if (!ready) {
                        stop = true;
                        break;
                    }
                }
                const uint32_t m = k >= g.cpr ? 1u : 0u;
                const uint32_t kc = k - m * g.cpr;
                uint32_t bytes;
                const uint16_t *src;
                if (g.parts == 1) {
                    const uint32_t rows = min(g.rpc, g.n - kc * g.rpc);
                    bytes = rows * g.cols * 2;
                    src = g.w + (static_cast<uint64_t>(g.u0) + kc * g.rpc + static_cast<uint64_t>(m) * g.units) * g.cols;
                } else {
                    bytes = ((kc & 1u) ? g.slots - kPtStageSubs : kPtStageSubs) * kSubElems * 2;
                    src = g.w + (static_cast<uint64_t>(g.u0) + (kc >> 1) + static_cast<uint64_t>(m) * g.units) * g.cols +
                          (kc & 1u) * (kPtStageSubs * kSubElems);
                }
                // Several copies in flight per stage: the copy engine moves more
                // bytes per SM with smaller, concurrent bulk copies.
                mbar_expect_tx(&full_bar[s], bytes);
                unsigned char *dst = ring + static_cast<size_t>(s) * kPtStageBytes;
                for (uint32_t off = 0; off < bytes; off += p.piece)
                    bulk_load(dst + off, reinterpret_cast<const unsigned char *>(src) + off, min(p.piece, bytes - off),
                              &full_bar[s], policy);
                if (p.trace && blockIdx.x == 0 && k == 0) p.trace[1 + (5 * p.L + 1) + ph] = global_ns();
                ++issued;
            }
        }
        // Every copy that was issued lands before the CTA exits, also when the
        // consumers stopped early (on the normal path they are landed or
        // about to be, since the consumers wait for each of them).
        (void)stop;
        for (uint32_t i = issued > stages ? issued - stages : 0; i < issued; ++i)
            mbar_wait(&full_bar[i % stages], (i / stages) & 1u);
        return;
    }

    // Consumers.
    uint32_t chunk = 0;
    int s = 0;
    float *xs = work;
    float *partial = work + ((p.H + 3) & ~3u);
    bool ok = true;
    for (uint32_t l = 0; l < p.L && ok; ++l) {
        const PtLayer &L = p.layers[l];
        // qkv projection, input: embedding (layer 0) or state + post-MLP branch.
        if (l == 0) {
            const uint32_t token = *p.token;
            if (pt_sync_any(token >= p.vocab)) {
                if (threadIdx.x == 0) pt_fail(p, 1u, abort_flag);
                ok = false;
                break;
            }
            pt_norm_input(p, token, true, nullptr, nullptr, nullptr, 0.0f, L.pre, 1.0f, p.state[0], nullptr, xs,
                          red);
        } else {
            if (!pt_grid_sync(p, gen, 5 * (l - 1) + 4, B, abort_flag)) {
                ok = false;
                break;
            }
            pt_norm_input(p, 0, false, s ? p.state[1] : p.state[0], p.branch, p.layers[l - 1].mpost, kPtPostMlp,
                          L.pre, 1.0f, s ? p.state[0] : p.state[1], nullptr, xs, red);
            s ^= 1;
        }
        const PtGemv gq = pt_gemv(p, 4 * l);
        chunk = pt_stream(p, gq, xs, nullptr, ring, full_bar, empty_bar, chunk, partial, abort_flag);
        if (chunk == kPtAbort) {
            ok = false;
            break;
        }
        pt_store_epilogue(gq, partial, p.qkv);
        if (!pt_grid_sync(p, gen, 5 * l, B, abort_flag)) {
            ok = false;
            break;
        }
        pt_attention(p, l, work);
        if (!pt_grid_sync(p, gen, 5 * l + 1, B, abort_flag)) {
            ok = false;
            break;
        }
        const PtGemv go = pt_gemv(p, 4 * l + 1);
        chunk = pt_stream(p, go, nullptr, p.attn, ring, full_bar, empty_bar, chunk, partial, abort_flag);
        if (chunk == kPtAbort) {
            ok = false;
            break;
        }
        pt_store_epilogue(go, partial, p.branch);
        if (!pt_grid_sync(p, gen, 5 * l + 2, B, abort_flag)) {
            ok = false;
            break;
        }
        pt_norm_input(p, 0, false, s ? p.state[1] : p.state[0], p.branch, L.post, kPtPostMixer, L.mpre, 1.0f,
                      s ? p.state[0] : p.state[1], nullptr, xs, red);
        s ^= 1;
        const PtGemv gg = pt_gemv(p, 4 * l + 2);
        chunk = pt_stream(p, gg, xs, nullptr, ring, full_bar, empty_bar, chunk, partial, abort_flag);
        if (chunk == kPtAbort) {
            ok = false;
            break;
        }
        pt_swiglu_epilogue(gg, partial, p.mid);
        if (!pt_grid_sync(p, gen, 5 * l + 3, B, abort_flag)) {
            ok = false;
            break;
        }
        const PtGemv gd = pt_gemv(p, 4 * l + 3);
        chunk = pt_stream(p, gd, nullptr, p.mid, ring, full_bar, empty_bar, chunk, partial, abort_flag);
        if (chunk == kPtAbort) {
            ok = false;
            break;
        }
        pt_store_epilogue(gd, partial, p.branch);
    }
    if (!ok || !pt_grid_sync(p, gen, 5 * (p.L - 1) + 4, B, abort_flag)) return;
    // Head: final norm of state + post-MLP branch, logits and candidates.
    pt_norm_input(p, 0, false, s ? p.state[1] : p.state[0], p.branch, p.layers[p.L - 1].mpost, kPtPostMlp, p.norm,
                  1.0f, s ? p.state[0] : p.state[1], p.normalized, xs, red);
    const PtGemv gh = pt_gemv(p, 4 * p.L);
    if (pt_stream(p, gh, xs, nullptr, ring, full_bar, empty_bar, chunk, partial, abort_flag) == kPtAbort) return;
    pt_head_epilogue(p, gh, partial, p.logits);
    // Only block 0 waits for every block's candidates.
    pt_consumer_sync();
    if (threadIdx.x == 0 && !*abort_flag) {
        __threadfence();
        red_release_gpu_add(p.bar, 1ull);
    }
    if (blockIdx.x != 0) return;
    if (threadIdx.x == 0 && !*abort_flag) {
        const unsigned long long target = (gen * B + B) * gridDim.x;
        const uint64_t start = global_ns();
        while (ld_acquire_gpu_u64(p.bar) < target) {
            if (pt_failed(p)) {
                *abort_flag = 1;
                break;
            }
            if (global_ns() - start > kPtWaitNs) {
                pt_fail(p, 5u, abort_flag);
                break;
            }
        }
        __threadfence();
        if (p.trace) p.trace[B] = global_ns();
    }
    if (pt_sync_any(*abort_flag) || warp != 0) return;
    // Merge the candidates (argmax_merge_kernel's rule), publish the token,
    // advance the committed rows and the launch generation.
    const float ninf = -__int_as_float(0x7f800000);
    float bv = ninf, sv = ninf;
    uint32_t bi = 0xffffffffu, nan_seen = 0;
    for (uint32_t b = lane; b < gridDim.x; b += 32) {
        nan_seen |= __ldcg(p.arg_nan + b);
        top2_merge(__ldcg(p.arg_val + b), __ldcg(p.arg_idx + b), __ldcg(p.arg_val2 + b), bv, bi, sv);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        const float os = __shfl_xor_sync(0xffffffffu, sv, o);
        nan_seen |= __shfl_xor_sync(0xffffffffu, nan_seen, o);
        top2_merge(ov, oi, os, bv, bi, sv);
    }
    for (uint32_t i = lane; i < p.L; i += 32) p.appended[i] += 1;
    if (lane == 0) {
        const uint32_t result = nan_seen ? 0xffffffffu : bi;
        p.next[0] = result;
        *p.token = result;
        p.next[2] = __float_as_uint(__fsub_rn(bv, sv));
        *p.gen = gen + 1;
    }
}

}  // namespace plamo
