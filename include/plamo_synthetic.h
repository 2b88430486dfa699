/* Seeded synthetic weights and activations, bit-identical on host and device.
 *
 * Checkpoints are not available on the benchmark hosts, so weights are drawn
 * from a counter-based generator instead: value(i) = mean + std * z(seed, i)
 * with z an Irwin-Hall sum of twelve uniform bytes, (S - 1530) / 256, which has
 * mean 0 and variance 65535/65536 and so stands in for N(0, 1) on [-5.98, 5.98].
 * Every step is an exact integer operation or one correctly rounded FP32
 * operation, so the CUDA fill kernel and this host version produce the same
 * bits, and a 16 GB model is generated in HBM in milliseconds instead of being
 * written, read and uploaded.
 */
#ifndef PLAMO_SYNTHETIC_H
#define PLAMO_SYNTHETIC_H
#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define PLAMO_HD __host__ __device__ __forceinline__
#else
#define PLAMO_HD static inline
#endif

PLAMO_HD uint64_t plamo_splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

/* z(seed, i) in steps of 1/256. */
PLAMO_HD float plamo_synthetic_z(uint64_t seed, uint64_t i) {
    uint64_t key = seed * 0xD1B54A32D192ED03ull;
    uint64_t a = plamo_splitmix64(key + 2 * i), b = plamo_splitmix64(key + 2 * i + 1);
    int sum = 0;
    for (int k = 0; k < 8; ++k)
        sum += (int)((a >> (8 * k)) & 0xff);
    for (int k = 0; k < 4; ++k)
        sum += (int)((b >> (8 * k)) & 0xff);
    return (float)(sum - 1530) * 0.00390625f;
}

PLAMO_HD float plamo_synthetic_f32(uint64_t seed, uint64_t i, float mean, float std) {
#if defined(__CUDA_ARCH__)
    return __fadd_rn(mean, __fmul_rn(std, plamo_synthetic_z(seed, i)));
#else
    volatile float product = std * plamo_synthetic_z(seed, i); /* one rounding, never fused */
    return mean + product;
#endif
}

/* Round-to-nearest-even FP32 -> BF16 bit pattern (finite inputs). */
PLAMO_HD uint16_t plamo_bf16_round(float value) {
    uint32_t bits;
    memcpy(&bits, &value, 4);
    bits += 0x7FFFu + ((bits >> 16) & 1u);
    return (uint16_t)(bits >> 16);
}

PLAMO_HD uint16_t plamo_synthetic_bf16(uint64_t seed, uint64_t i, float mean, float std) {
    return plamo_bf16_round(plamo_synthetic_f32(seed, i, mean, std));
}

#undef PLAMO_HD
#endif
