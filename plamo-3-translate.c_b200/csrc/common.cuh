// Shared device helpers of the PLaMo-3 sm_100a kernels.
//
// The library is compiled with --fmad=false: a multiply followed by an add is
// two rounded operations unless the source writes fmaf(). That keeps every
// elementwise formula in the same rounding order as the reference
// (RMSNorm (x*inv)*(w+offset), split-half RoPE with separate products, SwiGLU
// g/(exp(-g)+1)*u), while the long reductions (dot products, sums of squares,
// softmax sums) use parallel trees whose results stay within the reference's
// own GPU acceptance bound (relative L2 <= 1e-4).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace plamo {

constexpr int kWarp = 32;

__device__ __forceinline__ float bf16_to_f32(uint16_t bits) {
    return __uint_as_float(static_cast<uint32_t>(bits) << 16);
}
// Low/high BF16 of a packed 32-bit word -> FP32 (exact).
__device__ __forceinline__ float bf16_lo(uint32_t word) { return __uint_as_float(word << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t word) { return __uint_as_float(word & 0xFFFF0000u); }

// exp as the reference computes it (reference src/activation.s:6-46):
// saturate below -87 to 0 and above 88 to +inf, n = rint(x*log2e),
// r = fma(-n, ln2, x), degree-7 Taylor polynomial in FMA Horner form, times 2^n.
// Bit-identical to the C oracle's plamo_exp.
__device__ __forceinline__ float plamo_exp(float x) {
    if (!(x >= -87.0f)) return 0.0f;
    if (x > 88.0f) return __int_as_float(0x7f800000);
    float n = rintf(__fmul_rn(x, 1.4426950408889634f));
    int e = static_cast<int>(n);
    float r = fmaf(-n, 0.6931471805599453f, x);
    float p = 0.0001984126984126984f;
    p = fmaf(p, r, 0.001388888888888889f);
    p = fmaf(p, r, 0.008333333333333333f);
    p = fmaf(p, r, 0.041666666666666664f);
    p = fmaf(p, r, 0.16666666666666666f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    return __fmul_rn(p, __int_as_float((e + 127) << 23));
}

// SiLU(g) * u with the reference's operation order (src/activation.s:182-226).
__device__ __forceinline__ float swiglu(float g, float u) {
    float d = __fadd_rn(plamo_exp(-g), 1.0f);
    return __fmul_rn(__fdiv_rn(g, d), u);
}

__device__ __forceinline__ float4 ld4(const float *p) { return *reinterpret_cast<const float4 *>(p); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Deterministic block sum (same order for every block of the same shape).
// `scratch` holds at least blockDim.x/32 floats. All threads get the result.
__device__ __forceinline__ float block_sum(float v, float *scratch) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = (blockDim.x + 31) >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float total = 0.0f;
    for (int i = 0; i < warps; ++i) total += scratch[i];
    return total;
}

// RMSNorm inverse 1/sqrt(sum/n + 1e-6) from a sum of squares (reference
// src/math.s:349-366: divide, add eps, sqrt, reciprocal, each rounded).
__device__ __forceinline__ float rms_inverse(float sum_squares, uint64_t n) {
    // For a power-of-two n the product by the exact reciprocal is the same
    // correctly rounded quotient, without the division's latency.
    float mean = (n & (n - 1)) == 0 ? __fmul_rn(sum_squares, 1.0f / static_cast<float>(n))
                                    : __fdiv_rn(sum_squares, static_cast<float>(n));
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, 1e-6f)));
}
// (x * inverse) * (w + offset)
__device__ __forceinline__ float rms_apply(float x, float inverse, uint16_t w, float offset) {
    return __fmul_rn(__fmul_rn(x, inverse), __fadd_rn(bf16_to_f32(w), offset));
}

__device__ __forceinline__ float4 norm4(uint2 w, float offset) {
    return make_float4(__fadd_rn(bf16_lo(w.x), offset), __fadd_rn(bf16_hi(w.x), offset),
                       __fadd_rn(bf16_lo(w.y), offset), __fadd_rn(bf16_hi(w.y), offset));
}
__device__ __forceinline__ float sq4(float4 v) { return v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w; }
__device__ __forceinline__ float4 apply4(float4 x, float inv, float4 w) {
    return make_float4(__fmul_rn(__fmul_rn(x.x, inv), w.x), __fmul_rn(__fmul_rn(x.y, inv), w.y),
                       __fmul_rn(__fmul_rn(x.z, inv), w.z), __fmul_rn(__fmul_rn(x.w, inv), w.w));
}

// Streaming 128-bit load of weights that are read once per token: bypass L1
// and mark the L2 line evict-first so activations and KV stay resident.
__device__ __forceinline__ uint64_t evict_first_policy() {
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}
// A small, hot table read once per launch (KV page bases): keep its lines in
// L2 past the weight streams, which are marked evict-first.
__device__ __forceinline__ uint64_t evict_last_policy() {
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}
__device__ __forceinline__ uint64_t load_u64_keep(const void *p, uint64_t policy) {
    uint64_t v;
    asm volatile("ld.global.L2::cache_hint.u64 %0, [%1], %2;" : "=l"(v) : "l"(p), "l"(policy));
    return v;
}
__device__ __forceinline__ uint4 load_stream(const void *p, uint64_t policy) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p), "l"(policy));
    return v;
}

// Programmatic dependent launch: let the next kernel in the stream start its
// weight prefetch while this one finishes; wait for the previous kernel's
// results before reading them.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// ---- mbarrier + bulk async copy (TMA unit, no tensor map, no multicast) ----
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Launch timeline of a traced decode step: one record of kTraceWords words
// per traced launch, all starting at zero; minima are kept as UINT64_MAX - t
// so that every field is an atomicMax: [0] first CTA entry, [1] last CTA past
// its dependency wait and prologue, [2] first CTA done streaming, [3] last,
// [4] last CTA past the dependency wait alone, [5] last CTA entry.
constexpr int kTraceWords = 6;
__device__ __forceinline__ void trace_stamp(unsigned long long *rec, int field, uint64_t t) {
    if (field == 0 || field == 2) atomicMax(rec + field, ~0ull - t);
    else atomicMax(rec + field, static_cast<unsigned long long>(t));
}

// Wait for the phase of `parity` to complete, giving up after ~2 s of wall
// time (returns false; the caller records an error and drains).
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t start = global_ns();
    while (!mbar_try_wait(bar, parity))
        if (global_ns() - start > 2000000000ull) return false;
    return true;
}
// 1-D bulk copy global -> shared (16-byte aligned addresses, size multiple of
// 16), completion signalled as transaction bytes on `bar`, L2 evict-first.
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                          uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// 16-byte asynchronous global -> shared copy (LDGSTS), no registers involved.
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// Wait until at most one committed group (the newest) is still in flight.
__device__ __forceinline__ void cp_async_wait_one() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

}  // namespace plamo
