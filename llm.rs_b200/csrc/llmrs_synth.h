/*
 * llmrs_synth.h - seeded, counter-based synthetic model generator.
 *
 * One header, compiled three ways: by nvcc for device code (weight generation
 * kernels), by nvcc's host compiler (model set-up) and by gcc for the CPU
 * oracle.  Every value is produced by integer arithmetic plus at most two
 * correctly rounded f32 operations (no FMA), so the host and the device produce
 * bit-identical weights, activations and KV entries for the same
 * (seed, layer, tensor, index).
 *
 * Recipe (matches the synthetic models that the batch-1 token-loop configs
 * describe):
 *   - stream seed  : mix64(seed ^ layer<<32 ^ tensor<<8 ^ 0x1234)
 *   - i-th draw    : mix64(stream + (i+1) * golden_gamma)       (SplitMix64)
 *   - normal(0,1)  : Irwin-Hall sum of twelve 16-bit uniforms, centred and
 *                    divided by 65536 (exact in f32; support +-6 sigma)
 *   - Q4 codes     : uniform bytes (two uniform nibbles 0..15 per byte)
 *   - Q4/Q8 scales : f16_rne(|z| * 0.0025f) == fp16(|N(0,0.02)|/8), widened to
 *                    f32 (exactly representable)
 *   - Q8 codes     : ((u16 * 255) >> 16) - 127, i.e. -127..127
 *   - embeddings / norm weights : 1 + 0.02 z ;  activations / KV : z
 */
#ifndef LLMRS_SYNTH_H
#define LLMRS_SYNTH_H

#include <stdint.h>

#if defined(__CUDACC__)
#define LLMRS_HD __host__ __device__ __forceinline__
#else
#define LLMRS_HD static inline
#endif

#if defined(__CUDA_ARCH__)
#define LLMRS_FMUL(a, b) __fmul_rn((a), (b))
#define LLMRS_FADD(a, b) __fadd_rn((a), (b))
#else
/* host code is compiled with -ffp-contract=off; these are single roundings */
#define LLMRS_FMUL(a, b) ((a) * (b))
#define LLMRS_FADD(a, b) ((a) + (b))
#endif

#define LLMRS_GAMMA 0x9E3779B97F4A7C15ULL

/* tensor identifiers of the synthetic model (stream selectors) */
enum llmrs_synth_tensor {
    LLMRS_T_EMBED = 1,
    LLMRS_T_LM_HEAD = 2,
    LLMRS_T_FINAL_NORM = 3,
    LLMRS_T_TOKENS = 4,
    LLMRS_T_ACT = 5,
    LLMRS_T_ATTN_NORM = 10,
    LLMRS_T_Q = 11,
    LLMRS_T_K = 12,
    LLMRS_T_V = 13,
    LLMRS_T_O = 14,
    LLMRS_T_MLP_NORM = 15,
    LLMRS_T_GATE = 16,
    LLMRS_T_UP = 17,
    LLMRS_T_DOWN = 18,
    LLMRS_T_KCACHE = 19,
    LLMRS_T_VCACHE = 20
};
/* sub-streams of one quantised tensor */
enum { LLMRS_SUB_Q4CODES = 0, LLMRS_SUB_SCALES = 1, LLMRS_SUB_Q8CODES = 2, LLMRS_SUB_F32 = 3 };
/* layer index used for tensors that do not belong to a block */
#define LLMRS_GLOBAL_LAYER 0xFFFFu

LLMRS_HD uint64_t llmrs_mix64(uint64_t z)
{
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

LLMRS_HD uint64_t llmrs_stream(uint64_t seed, uint32_t layer, uint32_t tensor, uint32_t sub)
{
    return llmrs_mix64(seed ^ ((uint64_t)layer << 32) ^ ((uint64_t)(tensor * 4u + sub) << 8) ^ 0x1234ULL);
}

LLMRS_HD uint64_t llmrs_draw(uint64_t stream, uint64_t i)
{
    return llmrs_mix64(stream + (i + 1) * LLMRS_GAMMA);
}

LLMRS_HD int llmrs_sum4_u16(uint64_t r)
{
    return (int)(r & 0xFFFF) + (int)((r >> 16) & 0xFFFF) + (int)((r >> 32) & 0xFFFF) + (int)(r >> 48);
}

/* approximately N(0,1); exact in f32 */
LLMRS_HD float llmrs_normal(uint64_t stream, uint64_t i)
{
    int s = llmrs_sum4_u16(llmrs_draw(stream, 3 * i)) + llmrs_sum4_u16(llmrs_draw(stream, 3 * i + 1)) +
            llmrs_sum4_u16(llmrs_draw(stream, 3 * i + 2));
    return LLMRS_FMUL((float)(s - 393210), 1.0f / 65536.0f);
}

/* mu + sd * z, two correctly rounded operations */
LLMRS_HD float llmrs_normal_ms(uint64_t stream, uint64_t i, float mu, float sd)
{
    return LLMRS_FADD(mu, LLMRS_FMUL(sd, llmrs_normal(stream, i)));
}

LLMRS_HD uint32_t llmrs_f32_bits(float f)
{
    union { float f; uint32_t u; } c;
    c.f = f;
    return c.u;
}

LLMRS_HD float llmrs_bits_f32(uint32_t u)
{
    union { float f; uint32_t u; } c;
    c.u = u;
    return c.f;
}

/* IEEE binary32 -> binary16, round to nearest even, subnormals and overflow handled */
LLMRS_HD uint16_t llmrs_f32_to_f16(float f)
{
    uint32_t x = llmrs_f32_bits(f);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) /* inf / nan */
        return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
    if (ax >= 0x477FF000u) /* rounds to >= 65520 -> inf */
        return (uint16_t)(sign | 0x7C00u);
    if (ax < 0x38800000u) { /* result is subnormal or zero in f16 */
        if (ax < 0x33000000u) /* < 2^-25 rounds to zero */
            return (uint16_t)sign;
        uint32_t e = ax >> 23;          /* 102..112 */
        uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
        uint32_t shift = 126u - e;      /* 14..24 */
        uint32_t q = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (q & 1u)))
            q++;
        return (uint16_t)(sign | q);
    }
    /* normal */
    uint32_t q = ((ax >> 13) - (112u << 10));
    uint32_t rem = ax & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u)))
        q++;
    return (uint16_t)(sign | q);
}

LLMRS_HD float llmrs_f16_to_f32(uint16_t h)
{
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = ((uint32_t)h >> 10) & 0x1Fu;
    uint32_t m = (uint32_t)h & 0x3FFu;
    if (e == 0) {
        if (m == 0)
            return llmrs_bits_f32(sign);
        /* subnormal: m * 2^-24, exact in f32 */
        float v = LLMRS_FMUL((float)m, 1.0f / 16777216.0f);
        return sign ? -v : v;
    }
    if (e == 31)
        return llmrs_bits_f32(sign | 0x7F800000u | (m << 13));
    return llmrs_bits_f32(sign | ((e + 112u) << 23) | (m << 13));
}

/* block scale of a synthetic quantised weight, as f16 bits */
LLMRS_HD uint16_t llmrs_synth_scale_f16(uint64_t stream, uint64_t i)
{
    float z = llmrs_normal(stream, i);
    float a = z < 0.0f ? -z : z;
    return llmrs_f32_to_f16(LLMRS_FMUL(a, 0.0025f));
}

/* byte j of a synthetic planar Q4 nibble array (both nibbles uniform 0..15) */
LLMRS_HD uint8_t llmrs_synth_q4_byte(uint64_t stream, uint64_t j)
{
    return (uint8_t)(llmrs_draw(stream, j >> 3) >> ((j & 7u) * 8u));
}

/* element j of a synthetic Q8_0 code array, uniform in -127..127 */
LLMRS_HD int8_t llmrs_synth_q8_code(uint64_t stream, uint64_t j)
{
    uint32_t u = (uint32_t)(llmrs_draw(stream, j >> 2) >> ((j & 3u) * 16u)) & 0xFFFFu;
    return (int8_t)((int)((u * 255u) >> 16) - 127);
}

/* KV pre-fill element index: independent of how many positions are filled */
LLMRS_HD uint64_t llmrs_kv_index(uint32_t kv_head, uint32_t pos, uint32_t d, uint32_t head_dim)
{
    return ((uint64_t)kv_head << 40) | ((uint64_t)pos * head_dim + d);
}

#endif /* LLMRS_SYNTH_H */
