// Tensor-parallel exchange over peer memory (NVLink P2P through CUDA IPC
// mappings; plain loads and stores, no multicast, no library collective).
//
// A tensor-parallel PLaMo-3 block ends in a row-split projection (o_proj over
// this rank's heads, down_proj over this rank's MLP rows) whose output is a
// partial sum of the hidden vector. Every rank owns an exchange buffer; for
// each exchange point it holds one partial vector per source rank and one
// flag per source rank. The producing projection stores its output rows
// straight into slot `rank` of every peer's buffer (its own included) from
// its epilogue, so the transfer overlaps the rest of the projection; the last
// CTA to finish raises this rank's flag at every peer. The consuming kernel
// (the next projection's prologue, or a row kernel for prompts) waits for
// every rank's flag of the current epoch and sums the partials in rank order,
// so every rank computes the same bits.
//
// Decode points use a low-latency form instead of flags: every partial value
// travels with its epoch tag in one aligned 64-bit word (value bits in the low
// half, epoch + 1 in the high half), written with one scalar 64-bit relaxed
// system-scope store and read with loads whose elements are 64-bit words
// (scalar, or a v2.u64 vector, which the PTX memory model treats as two
// 64-bit element accesses). An aligned 64-bit access is single-copy atomic,
// so a reader that sees the new tag also sees the value stored with it; the
// consumer polls the values themselves and proceeds the moment the last one
// lands - no fence, ticket or flag round trip on the producer side.
//
// Epochs: a device counter, advanced once at the end of every tensor-parallel
// operation (decode step, prompt, verification) on every rank; a flag holds
// epoch + 1 of the operation that raised it, so buffers and flags are reused
// without resets. Every wait is bounded (2 s of %globaltimer): on timeout the
// kernel records error 4 and continues with whatever is in the buffer. Once
// error 4 is recorded, the rest of the operation neither waits nor writes to
// peers: a peer that stopped (or whose process is exiting) is left alone
// within 2 s, and its memory is not touched after that.
#pragma once
#include "common.cuh"

namespace plamo {

constexpr int kTpMax = 8;

struct TpPoint {
    uint32_t tp;                    // ranks; 0 = not tensor-parallel
    uint32_t ll;                    // 1: parts hold {value, tag} pairs, no flags
    uint64_t stride;                // elements between source slots of `parts`
    const float *parts;             // local [tp][stride] partials, slot r from rank r
    const uint32_t *flags;          // local [tp] flag raised by each source rank
    float *peer_parts[kTpMax];      // slot `rank` of every rank's parts
    uint32_t *peer_flags[kTpMax];   // flag `rank` of every rank's flags
    uint32_t *ticket;               // local CTA arrival counter of this point
    const uint32_t *epoch;          // local epoch counter
    uint32_t *error;                // set to 4 when a peer never arrived
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// One thread: wait until every rank's flag of this point shows the current
// epoch. Returns false after ~2 s (error recorded).
__device__ __forceinline__ bool tp_failed(const uint32_t *error) {
    return error && *reinterpret_cast<const volatile uint32_t *>(error) == 4u;
}

__device__ __forceinline__ bool tp_wait_flags(const TpPoint &t) {
    if (tp_failed(t.error)) return false;
    const uint32_t want = *t.epoch + 1;
    uint64_t start = 0;
    for (uint32_t r = 0; r < t.tp; ++r) {
        while (ld_acquire_sys(t.flags + r) != want) {
            if (!start) start = global_ns();
            else if (global_ns() - start > 2000000000ull) {
                if (t.error) atomicExch(t.error, 4u);
                return false;
            }
        }
    }
    return true;
}

// Called by every thread of a producing CTA after its stores to the peers:
// the last CTA of the grid raises this rank's flag at every peer, one thread
// per peer (fence, then the flag), so the peers are signalled concurrently.
__device__ __forceinline__ void tp_signal(const TpPoint &t) {
    __shared__ uint32_t last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        last = atomicAdd(t.ticket, 1u) == gridDim.x - 1;
        if (last) *t.ticket = 0;
    }
    __syncthreads();
    if (last && threadIdx.x < t.tp && !tp_failed(t.error)) {
        __threadfence_system();
        st_relaxed_sys(t.peer_flags[threadIdx.x], *t.epoch + 1);
    }
}

// Tagged words of the low-latency points: {value bits, tag} as one 64-bit
// word. Two consecutive words per load (16-byte aligned); each element is
// a 64-bit access of its own.
__device__ __forceinline__ ulonglong2 ld_tagged2(const void *p) {
    ulonglong2 v;
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0,%1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint64_t ld_tagged1(const void *p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_tagged(void *p, float value, uint32_t tag) {
    const uint64_t word = static_cast<uint64_t>(__float_as_uint(value)) | (static_cast<uint64_t>(tag) << 32);
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(word) : "memory");
}
__device__ __forceinline__ uint32_t tag_of(uint64_t word) { return static_cast<uint32_t>(word >> 32); }
__device__ __forceinline__ float value_of(uint64_t word) { return __uint_as_float(static_cast<uint32_t>(word)); }

// Low-latency point: this rank's value of element `unit` to every rank.
__device__ __forceinline__ void tp_ll_store(const TpPoint &t, uint64_t unit, float v, uint32_t tag) {
    for (uint32_t r = 0; r < t.tp; ++r) st_tagged(reinterpret_cast<uint64_t *>(t.peer_parts[r]) + unit, v, tag);
}

// Wait (bounded) until `ok(...)` holds for the polled words; false on timeout
// or an earlier failure of this operation.
template <typename Load, typename Ready>
__device__ __forceinline__ bool tp_ll_poll(const TpPoint &t, Load load, Ready ready, uint64_t &start) {
    for (;;) {
        load();
        if (ready()) return true;
        if (tp_failed(t.error)) return false;
        if (!start) start = global_ns();
        else if (global_ns() - start > 2000000000ull) {
            if (t.error) atomicExch(t.error, 4u);
            return false;
        }
    }
}

// Rank-ordered sums of KP groups of 4 elements (group k at element
// 4 * (i0 + k * step), present when below n4) of a low-latency point: the
// loads of all groups of one rank are in flight together, so a rank costs
// one round trip once its values have landed (not one per group).
template <int KP>
__device__ __forceinline__ void tp_ll_sum_groups(const TpPoint &t, uint32_t i0, uint32_t step, uint32_t n4,
                                                 uint32_t tag, float4 (&out)[KP]) {
    uint64_t start = 0;
    for (uint32_t r = 0; r < t.tp; ++r) {
        const uint64_t *slot = reinterpret_cast<const uint64_t *>(t.parts) + r * t.stride;
        ulonglong2 a[KP], b[KP];
        uint32_t pending = 0;
#pragma unroll
        for (int k = 0; k < KP; ++k)
            if (i0 + k * step < n4) pending |= 1u << k;
        const uint32_t present = pending;
        while (pending) {
#pragma unroll
            for (int k = 0; k < KP; ++k)
                if (pending >> k & 1u) {
                    const uint64_t *src = slot + 4ull * (i0 + k * step);
                    a[k] = ld_tagged2(src);
                    b[k] = ld_tagged2(src + 2);
                }
#pragma unroll
            for (int k = 0; k < KP; ++k)
                if ((pending >> k & 1u) && tag_of(a[k].x) == tag && tag_of(a[k].y) == tag &&
                    tag_of(b[k].x) == tag && tag_of(b[k].y) == tag)
                    pending &= ~(1u << k);
            if (!pending || tp_failed(t.error)) break;
            if (!start) start = global_ns();
            else if (global_ns() - start > 2000000000ull) {
                if (t.error) atomicExch(t.error, 4u);
                break;
            }
        }
#pragma unroll
        for (int k = 0; k < KP; ++k)
            if (present >> k & 1u) {
                const float4 v = make_float4(value_of(a[k].x), value_of(a[k].y), value_of(b[k].x), value_of(b[k].y));
                out[k] = r ? make_float4(__fadd_rn(out[k].x, v.x), __fadd_rn(out[k].y, v.y), __fadd_rn(out[k].z, v.z),
                                         __fadd_rn(out[k].w, v.w))
                           : v;
            }
    }
}

__device__ __forceinline__ float tp_ll_sum1(const TpPoint &t, uint64_t i, uint32_t tag) {
    float s = 0.0f;
    uint64_t start = 0;
    for (uint32_t r = 0; r < t.tp; ++r) {
        const uint64_t *src = reinterpret_cast<const uint64_t *>(t.parts) + r * t.stride + i;
        uint64_t a = 0;
        tp_ll_poll(t, [&] { a = ld_tagged1(src); }, [&] { return tag_of(a) == tag; }, start);
        s = r ? __fadd_rn(s, value_of(a)) : value_of(a);
    }
    return s;
}

// Rank-ordered sum of the 4 floats at `i` of every source slot (L2 loads:
// the rows arrive from other GPUs, L1 may hold the previous epoch's).
__device__ __forceinline__ float4 tp_sum4(const TpPoint &t, uint64_t i) {
    float4 s = __ldcg(reinterpret_cast<const float4 *>(t.parts + i));
    for (uint32_t r = 1; r < t.tp; ++r) {
        const float4 v = __ldcg(reinterpret_cast<const float4 *>(t.parts + r * t.stride + i));
        s = make_float4(__fadd_rn(s.x, v.x), __fadd_rn(s.y, v.y), __fadd_rn(s.z, v.z), __fadd_rn(s.w, v.w));
    }
    return s;
}
__device__ __forceinline__ float tp_sum1(const TpPoint &t, uint64_t i) {
    float s = __ldcg(t.parts + i);
    for (uint32_t r = 1; r < t.tp; ++r) s = __fadd_rn(s, __ldcg(t.parts + r * t.stride + i));
    return s;
}

// Prompt all-reduce, push half: copy n floats of this rank's partial rows
// into slot `rank` of every peer (n % 4 == 0, 16-byte aligned), then signal.
__global__ void tp_push_kernel(const float *src, uint64_t n, TpPoint t) {
    pdl_wait();
    const uint64_t n4 = tp_failed(t.error) ? 0 : n / 4;
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n4;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const float4 v = reinterpret_cast<const float4 *>(src)[i];
        for (uint32_t r = 0; r < t.tp; ++r) reinterpret_cast<float4 *>(t.peer_parts[r])[i] = v;
    }
    tp_signal(t);
}

// Prompt all-reduce, sum half: dst = rank-ordered sum of every slot.
__global__ void tp_sum_kernel(float *dst, uint64_t n, TpPoint t) {
    pdl_wait();
    if (threadIdx.x == 0) tp_wait_flags(t);
    __syncthreads();
    const uint64_t n4 = n / 4;
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n4;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x)
        reinterpret_cast<float4 *>(dst)[i] = tp_sum4(t, 4 * i);
    pdl_launch_dependents();
}

// Greedy token across the ranks' head slices. Slot layout per source rank:
// {value, global index, flag, pad}; index UINT32_MAX marks a NaN on that rank.
struct TpArg {
    uint32_t tp, rank;
    uint32_t *slots;            // local [rows][tp][4]
    uint32_t *peer_slots[kTpMax];  // every rank's [rows][tp][4] (slot `rank` is written)
    const uint32_t *epoch;
    uint32_t *error;
};

// rows = 1 (decode / prefill) or the candidates of a verification. Input:
// this rank's per-row best (value, local index) and the head slice offset.
// Output: the first maximal global index of every row, UINT32_MAX on NaN.
__global__ void tp_argmax_kernel(const float *val, const uint32_t *idx, uint32_t rows, uint32_t offset, TpArg a,
                                 uint32_t *out, uint32_t *next_token) {
    pdl_wait();
    const uint32_t flag = *a.epoch + 1;
    const bool failed = tp_failed(a.error);
    // One thread per (row, peer): value and index, fence, flag.
    for (uint32_t i = threadIdx.x; i < rows * a.tp && !failed; i += blockDim.x) {
        const uint32_t row = i / a.tp, r = i - row * a.tp;
        const uint32_t li = idx[row];
        uint32_t *s = a.peer_slots[r] + (static_cast<size_t>(row) * a.tp + a.rank) * 4;
        s[0] = __float_as_uint(val[row]);
        s[1] = li == 0xffffffffu ? li : li + offset;
        __threadfence_system();
        st_relaxed_sys(s + 2, flag);
    }
    __syncthreads();
    for (uint32_t row = threadIdx.x; row < rows; row += blockDim.x) {
        float bv = -__int_as_float(0x7f800000);
        uint32_t bi = 0xffffffffu;
        bool nan_seen = false;
        const uint64_t start = global_ns();
        for (uint32_t r = 0; r < a.tp && !failed; ++r) {
            const uint32_t *s = a.slots + (static_cast<size_t>(row) * a.tp + r) * 4;
            bool arrived = true;
            while (ld_acquire_sys(s + 2) != flag)
                if (global_ns() - start > 2000000000ull) {
                    if (a.error) atomicExch(a.error, 4u);
                    arrived = false;
                    break;
                }
            if (!arrived) {
                nan_seen = true;
                break;
            }
            const float v = __uint_as_float(__ldcg(s));
            const uint32_t i = __ldcg(s + 1);
            if (i == 0xffffffffu) nan_seen = true;
            else if (v > bv || (v == bv && i < bi)) {
                bv = v;
                bi = i;
            }
        }
        const uint32_t result = nan_seen ? 0xffffffffu : bi;
        out[row] = result;
        if (next_token) *next_token = result;
    }
}

// Advance the epoch (last kernel of every tensor-parallel operation).
__global__ void tp_epoch_kernel(uint32_t *epoch) {
    pdl_wait();
    if (threadIdx.x == 0) *epoch += 1;
}

}  // namespace plamo
