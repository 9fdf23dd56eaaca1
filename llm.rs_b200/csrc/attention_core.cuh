// attention_core.cuh - device pieces of batch-1 decode attention (attention.cu):
// the swizzled K-box layout, table-driven RoPE, and the per-warp chunk step
// (bit-exact scores, online softmax, V accumulation).
#pragma once

#include "common.cuh"

namespace llmrs {

namespace {

// K chunk in shared memory: the 3-D box [D/32 segments][CH rows][32 floats]
// with the 128-byte swizzle (16-byte unit u of 128-byte line L lands at unit
// u ^ (L % 8)), so lanes reading the same columns of 8 different rows hit 8
// different bank groups.  Float index of (row r, column d):
template <int CHR>
__device__ __forceinline__ int kswz(int r, int d)
{
    const int line = (d >> 5) * CHR + r;
    return line * 32 + ((((d >> 2) & 7) ^ (line & 7)) << 2) + (d & 3);
}

// cos/sin table values this lane needs for rotate-half RoPE (lane l holds
// dims l*DL.., frequency index (l % 16)*DL + k)
template <int D>
__device__ __forceinline__ void rope_table_lane(float (&c)[D / 32], float (&s)[D / 32], int lane, const float *cosr,
                                                const float *sinr)
{
    constexpr int DL = D / 32;
#pragma unroll
    for (int k = 0; k < DL; k++) {
        c[k] = cosr[(lane & 15) * DL + k];
        s[k] = sinr[(lane & 15) * DL + k];
    }
}

// rotate-half RoPE of one head held DL values per lane, exact reference
// arithmetic: x[j]*cos - x[j+mid]*sin ; x[j]*sin + x[j+mid]*cos
template <int D>
__device__ __forceinline__ void rope_lane(float (&x)[D / 32], int lane, const float (&c)[D / 32],
                                          const float (&s)[D / 32])
{
    constexpr int DL = D / 32;
    float other[DL];
#pragma unroll
    for (int k = 0; k < DL; k++)
        other[k] = __shfl_xor_sync(0xffffffffu, x[k], 16);
    const bool upper = lane >= 16;
#pragma unroll
    for (int k = 0; k < DL; k++) {
        if (!upper)
            x[k] = __fsub_rn(__fmul_rn(x[k], c[k]), __fmul_rn(other[k], s[k]));
        else
            x[k] = __fadd_rn(__fmul_rn(other[k], s[k]), __fmul_rn(x[k], c[k]));
    }
}

// DL consecutive floats of a shared-memory row (16- or 8-byte vector load)
template <int DL>
__device__ __forceinline__ void lds_lane(float (&r)[DL], const float *src)
{
    if constexpr (DL == 4) {
        const float4 t = *reinterpret_cast<const float4 *>(src);
        r[0] = t.x; r[1] = t.y; r[2] = t.z; r[3] = t.w;
    } else if constexpr (DL == 2) {
        const float2 t = *reinterpret_cast<const float2 *>(src);
        r[0] = t.x; r[1] = t.y;
    } else {
#pragma unroll
        for (int k = 0; k < DL; k++)
            r[k] = src[k];
    }
}

// One warp's step over 8 cached positions: rows row0 .. row0+7 of a K box of
// CHR rows (kbox, swizzled as kswz<CHR>) and the matching plain V rows vrows
// [8][D]; positions >= nvalid are masked.  Scores: lane owns (row b*G +
// lane/NREP, head lane%NREP) and sums q[d]*k[d] for d = 0..D-1 in order,
// unfused, like the reference's f32 dot (src/backend/cpu.rs:458-551, the
// non-aarch64 branch), then scales by 1/sqrt(D) (src/core/layer.rs:258):
// bit-exact scores.  Online softmax state: m_run / l_run of head lane%NREP;
// acc[h][k] = dims lane*DL+k of head h.  probs: this warp's [8*NREP] scratch.
template <int D, int NREP, int CHR>
__device__ __forceinline__ void attn_chunk(const float *kbox, int row0, const float *vrows, int nvalid,
                                           const float *q_s, int qstride, float *probs, float inv_sqrt_d,
                                           float &m_run, float &l_run, float (&acc)[NREP][D / 32], int lane)
{
    static_assert(CHR % 8 == 0, "K boxes are whole swizzle atoms");
    constexpr int DL = D / 32;
    constexpr int G = 32 / NREP; // positions per lane round
    constexpr int NFLY = 8 / G;
    float sc[NFLY];
    {
        const float *qh = q_s + (lane % NREP) * qstride;
        int roff[NFLY], rx[NFLY];
        float dot[NFLY];
#pragma unroll
        for (int b = 0; b < NFLY; b++) {
            const int r = row0 + b * G + lane / NREP;
            roff[b] = r * 32;
            rx[b] = r & 7;
            dot[b] = 0.0f;
        }
#pragma unroll
        for (int d4 = 0; d4 < D / 4; d4++) {
            const float4 qv = *reinterpret_cast<const float4 *>(qh + d4 * 4);
#pragma unroll
            for (int b = 0; b < NFLY; b++) {
                const float4 kv = *reinterpret_cast<const float4 *>(kbox + (d4 >> 3) * (CHR * 32) + roff[b] +
                                                                    (((d4 & 7) ^ rx[b]) << 2));
                float t = dot[b];
                t = __fadd_rn(t, __fmul_rn(qv.x, kv.x));
                t = __fadd_rn(t, __fmul_rn(qv.y, kv.y));
                t = __fadd_rn(t, __fmul_rn(qv.z, kv.z));
                t = __fadd_rn(t, __fmul_rn(qv.w, kv.w));
                dot[b] = t;
            }
        }
#pragma unroll
        for (int b = 0; b < NFLY; b++)
            sc[b] = (b * G + lane / NREP) < nvalid ? __fmul_rn(dot[b], inv_sqrt_d) : -INFINITY;
    }
    // lane holds (position b*G + lane/NREP, head lane%NREP) for each b
    float tmax = sc[0];
#pragma unroll
    for (int b = 1; b < NFLY; b++)
        tmax = fmaxf(tmax, sc[b]);
#pragma unroll
    for (int o = NREP; o < 32; o <<= 1)
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
    const float m_new = fmaxf(m_run, tmax);
    const float corr = (m_run == -INFINITY) ? 0.0f : expf(m_run - m_new);
    float psum = 0.0f;
#pragma unroll
    for (int b = 0; b < NFLY; b++) {
        const float pr = (sc[b] == -INFINITY) ? 0.0f : expf(sc[b] - m_new);
        probs[b * 32 + lane] = pr; // index position * NREP + head
        psum += pr;
    }
#pragma unroll
    for (int o = NREP; o < 32; o <<= 1)
        psum += __shfl_xor_sync(0xffffffffu, psum, o);
    l_run = l_run * corr + psum;
    m_run = m_new;
#pragma unroll
    for (int h = 0; h < NREP; h++) {
        const float ch = __shfl_sync(0xffffffffu, corr, h);
#pragma unroll
        for (int k = 0; k < DL; k++)
            acc[h][k] *= ch;
    }
    __syncwarp();
#pragma unroll
    for (int pl = 0; pl < 8; pl++) {
        if (pl < nvalid) {
            float vr[DL];
            lds_lane<DL>(vr, vrows + pl * D + lane * DL);
            float ph[NREP];
#pragma unroll
            for (int h4 = 0; h4 < NREP; h4 += 4) {
                const float4 t = *reinterpret_cast<const float4 *>(probs + pl * NREP + h4);
                ph[h4] = t.x;
                ph[h4 + 1] = t.y;
                ph[h4 + 2] = t.z;
                ph[h4 + 3] = t.w;
            }
#pragma unroll
            for (int h = 0; h < NREP; h++)
#pragma unroll
                for (int k = 0; k < DL; k++)
                    acc[h][k] = fmaf(ph[h], vr[k], acc[h][k]);
        }
    }
    __syncwarp();
}

// The new position (RoPE'd key knew and value vnew, plain [D] rows in shared
// memory), same arithmetic as attn_chunk with one valid row: lane h < NREP
// forms head h's score in order over d.
template <int D, int NREP>
__device__ __forceinline__ void attn_new_position(const float *knew, const float *vnew, const float *q_s, int qstride,
                                                  float inv_sqrt_d, float &m_run, float &l_run,
                                                  float (&acc)[NREP][D / 32], int lane)
{
    constexpr int DL = D / 32;
    float dot = 0.0f;
    if (lane < NREP) {
        const float *qh = q_s + lane * qstride;
        for (int d = 0; d < D; d++)
            dot = __fadd_rn(dot, __fmul_rn(qh[d], knew[d]));
        dot = __fmul_rn(dot, inv_sqrt_d);
    }
    const float sc = __shfl_sync(0xffffffffu, dot, lane % NREP); // score of head lane%NREP
    const float m_new = fmaxf(m_run, sc);
    const float corr = (m_run == -INFINITY) ? 0.0f : expf(m_run - m_new);
    const float pr = expf(sc - m_new);
    l_run = l_run * corr + pr;
    m_run = m_new;
    float vr[DL];
    lds_lane<DL>(vr, vnew + lane * DL);
#pragma unroll
    for (int h = 0; h < NREP; h++) {
        const float ch = __shfl_sync(0xffffffffu, corr, h);
        const float ph = __shfl_sync(0xffffffffu, pr, h);
#pragma unroll
        for (int k = 0; k < DL; k++)
            acc[h][k] = fmaf(ph, vr[k], acc[h][k] * ch);
    }
}

} // namespace

} // namespace llmrs
