// Block decoders (quant.rs:383-537, quant_iq.rs:409-426, 565-585, 732-754,
// 944-998, 1159-1189), shared by the decode kernels and by the encoders'
// fused error epilogue.  Every decoder keeps the reference's operand order,
// e.g. Q4_K (d*sc)*q - dmin*m and IQ2 ((d*(0.5+s))*0.25*g)*sign, so decoded
// values are bit-identical to decode_row.  The tables are per translation
// unit (no relocatable device code).
#pragma once
#include "iq_tables.h"
#include "kernels.cuh"

namespace shc {

static __device__ const uint8_t d_ksigns_iq2xs[128] = SH_KSIGNS_IQ2XS_DATA;
static __device__ const uint64_t d_iq2xxs_grid[256] = SH_IQ2XXS_GRID_DATA;
static __device__ const uint64_t d_iq2xs_grid[512] = SH_IQ2XS_GRID_DATA;
static __device__ const uint64_t d_iq2s_grid[1024] = SH_IQ2S_GRID_DATA;
static __device__ const uint32_t d_iq3xxs_grid[256] = SH_IQ3XXS_GRID_DATA;
static __device__ const uint32_t d_iq3s_grid[512] = SH_IQ3S_GRID_DATA;
static __device__ const int8_t d_kvalues_iq4nl[16] = SH_KVALUES_IQ4NL_DATA;

__device__ __forceinline__ float ldh(const uint8_t *p) { return f16_val((uint16_t)(p[0] | (p[1] << 8))); }
__device__ __forceinline__ uint32_t ldu32(const uint8_t *p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

// Decode elements [sub*32, sub*32+32) of one block of a block-quantized type.
__device__ __forceinline__ void decode_sub32(uint32_t type, const uint8_t *blk, int sub, float y[32]) {
    switch (type) {
    case SHC_TYPE_Q8_0: {
        const float d = ldh(blk);
#pragma unroll
        for (int j = 0; j < 32; j++) y[j] = d * (float)(int8_t)blk[2 + j];
        break;
    }
    case SHC_TYPE_Q4_0: {
        const float d = ldh(blk);
        const uint8_t *qs = blk + 2;
#pragma unroll
        for (int j = 0; j < 16; j++) {
            y[j] = d * (float)((int)(qs[j] & 0xF) - 8);
            y[16 + j] = d * (float)((int)(qs[j] >> 4) - 8);
        }
        break;
    }
    case SHC_TYPE_Q5_0: {
        const float d = ldh(blk);
        const uint32_t qh = ldu32(blk + 2);
        const uint8_t *qs = blk + 6;
#pragma unroll
        for (int j = 0; j < 16; j++) {
            const uint32_t q0 = (qs[j] & 0xFu) | (((qh >> j) & 1u) << 4);
            const uint32_t q1 = (uint32_t)(qs[j] >> 4) | (((qh >> (16 + j)) & 1u) << 4);
            y[j] = d * (float)((int)q0 - 16);
            y[16 + j] = d * (float)((int)q1 - 16);
        }
        break;
    }
    case SHC_TYPE_Q4_1: {
        const float d = ldh(blk), m = ldh(blk + 2);
        const uint8_t *qs = blk + 4;
#pragma unroll
        for (int j = 0; j < 16; j++) {
            y[j] = d * (float)(qs[j] & 0xF) + m;
            y[16 + j] = d * (float)(qs[j] >> 4) + m;
        }
        break;
    }
    case SHC_TYPE_Q5_1: {
        const float d = ldh(blk), m = ldh(blk + 2);
        const uint32_t qh = ldu32(blk + 4);
        const uint8_t *qs = blk + 8;
#pragma unroll
        for (int j = 0; j < 16; j++) {
            const uint32_t q0 = (qs[j] & 0xFu) | (((qh >> j) & 1u) << 4);
            const uint32_t q1 = (uint32_t)(qs[j] >> 4) | (((qh >> (16 + j)) & 1u) << 4);
            y[j] = d * (float)q0 + m;
            y[16 + j] = d * (float)q1 + m;
        }
        break;
    }
    case SHC_TYPE_Q6_K: {
        // elements h*128 + jj*32 + l
        const int h = sub >> 2, jj = sub & 3;
        const float d = ldh(blk + 208);
        const uint8_t *ql = blk + h * 64, *qh = blk + 128 + h * 32;
        const int8_t *sc = (const int8_t *)(blk + 192 + h * 8);
#pragma unroll
        for (int l = 0; l < 32; l++) {
            const int is = l / 16;
            int qv;
            if (jj == 0) qv = ((ql[l] & 0xF) | ((qh[l] & 3) << 4)) - 32;
            else if (jj == 1) qv = ((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
            else if (jj == 2) qv = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
            else qv = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
            y[l] = d * (float)sc[is + 2 * jj] * (float)qv;
        }
        break;
    }
    case SHC_TYPE_Q2_K: {
        // element sub*32 + l: sub-block 2*sub + l/16, 2-bit plane sub&3 of
        // byte 16 + (sub>>2)*32 + l; (d*sc)*q - dmin*m as ggml's dequantizer
        const float d = ldh(blk + 80), dmin = ldh(blk + 82);
        const uint8_t *qs = blk + 16 + (sub >> 2) * 32;
        const int shift = 2 * (sub & 3);
#pragma unroll
        for (int l = 0; l < 32; l++) {
            const uint8_t sc = blk[2 * sub + l / 16];
            const int qv = (qs[l] >> shift) & 3;
            y[l] = (d * (float)(sc & 0xF)) * (float)qv - dmin * (float)(sc >> 4);
        }
        break;
    }
    case SHC_TYPE_Q3_K: {
        // element sub*32 + l: 6-bit signed scale code of sub-block 2*sub + l/16,
        // low 2 bits in plane sub&3 of byte 32 + (sub>>2)*32 + l, high bit
        // sub of hmask byte l (a clear bit subtracts 4)
        const float d = ldh(blk + 108);
        const uint8_t *qs = blk + 32 + (sub >> 2) * 32;
        const int shift = 2 * (sub & 3);
#pragma unroll
        for (int l = 0; l < 32; l++) {
            const int sb = 2 * sub + l / 16;
            const int u = ((blk[96 + (sb & 7)] >> (4 * (sb >> 3))) & 0xF) | (((blk[104 + (sb & 3)] >> (2 * (sb >> 2))) & 3) << 4);
            const int lo = (qs[l] >> shift) & 3;
            const int hi = (blk[l] >> sub) & 1;
            y[l] = (d * (float)(u - 32)) * (float)(lo - (hi ? 0 : 4));
        }
        break;
    }
    case SHC_TYPE_Q4_K:
    case SHC_TYPE_Q5_K: {
        const bool five = type == SHC_TYPE_Q5_K;
        const float d = ldh(blk), dmin = ldh(blk + 2);
        const uint8_t *q = blk + 4;
        const int j = sub;
        uint8_t sc, m;
        if (j < 4) {
            sc = q[j] & 63;
            m = q[j + 4] & 63;
        } else {
            sc = (uint8_t)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
            m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
        }
        const float d1 = d * (float)sc, m1 = dmin * (float)m;
        const int chunk = sub >> 1, hi = sub & 1;
        const uint8_t *qs = blk + (five ? 48 : 16) + chunk * 32;
        if (five) {
            const uint8_t *qh = blk + 16;
            const uint8_t u = (uint8_t)(1u << sub);
#pragma unroll
            for (int l = 0; l < 32; l++) {
                const float qv = (float)(hi ? (qs[l] >> 4) : (qs[l] & 0xF)) + ((qh[l] & u) ? 16.0f : 0.0f);
                y[l] = d1 * qv - m1;
            }
        } else {
#pragma unroll
            for (int l = 0; l < 32; l++) y[l] = d1 * (float)(hi ? (qs[l] >> 4) : (qs[l] & 0xF)) - m1;
        }
        break;
    }
    case SHC_TYPE_IQ2_XXS: {
        const float d = ldh(blk);
        const uint32_t a0 = ldu32(blk + 2 + 8 * sub), a1 = ldu32(blk + 6 + 8 * sub);
        const float db = d * (0.5f + (float)(a1 >> 28)) * 0.25f;
#pragma unroll
        for (int l = 0; l < 4; l++) {
            const uint64_t g = d_iq2xxs_grid[(a0 >> (8 * l)) & 255];
            const uint8_t signs = d_ksigns_iq2xs[(a1 >> (7 * l)) & 127];
#pragma unroll
            for (int j = 0; j < 8; j++)
                y[8 * l + j] = db * (float)(uint8_t)(g >> (8 * j)) * ((signs >> j) & 1 ? -1.0f : 1.0f);
        }
        break;
    }
    case SHC_TYPE_IQ2_XS: {
        const float d = ldh(blk);
        const uint8_t sc = blk[66 + sub];
        const float db0 = d * (0.5f + (float)(sc & 0xF)) * 0.25f;
        const float db1 = d * (0.5f + (float)(sc >> 4)) * 0.25f;
#pragma unroll
        for (int l = 0; l < 4; l++) {
            const uint16_t qv = (uint16_t)(blk[2 + 8 * sub + 2 * l] | (blk[3 + 8 * sub + 2 * l] << 8));
            const uint64_t g = d_iq2xs_grid[qv & 511];
            const uint8_t signs = d_ksigns_iq2xs[qv >> 9];
            const float db = l < 2 ? db0 : db1;
#pragma unroll
            for (int j = 0; j < 8; j++)
                y[8 * l + j] = db * (float)(uint8_t)(g >> (8 * j)) * ((signs >> j) & 1 ? -1.0f : 1.0f);
        }
        break;
    }
    case SHC_TYPE_IQ2_S: {
        const float d = ldh(blk);
        const uint8_t *qs = blk + 2, *qh = blk + 66, *sc = blk + 74;
        const float db0 = d * (0.5f + (float)(sc[sub] & 0xF)) * 0.25f;
        const float db1 = d * (0.5f + (float)(sc[sub] >> 4)) * 0.25f;
#pragma unroll
        for (int l = 0; l < 4; l++) {
            const int idx = qs[4 * sub + l] | ((qh[sub] << (8 - 2 * l)) & 0x300);
            const uint64_t g = d_iq2s_grid[idx];
            const uint8_t signs = qs[32 + 4 * sub + l];
            const float db = l < 2 ? db0 : db1;
#pragma unroll
            for (int j = 0; j < 8; j++)
                y[8 * l + j] = db * (float)(uint8_t)(g >> (8 * j)) * ((signs >> j) & 1 ? -1.0f : 1.0f);
        }
        break;
    }
    case SHC_TYPE_IQ3_XXS: {
        const float d = ldh(blk);
        const uint8_t *qs = blk + 2;
        const uint32_t aux = ldu32(blk + 66 + 4 * sub);
        const float db = d * (0.5f + (float)(aux >> 28)) * 0.5f;
#pragma unroll
        for (int l = 0; l < 4; l++) {
            const uint8_t signs = d_ksigns_iq2xs[(aux >> (7 * l)) & 127];
            const uint32_t g1 = d_iq3xxs_grid[qs[8 * sub + 2 * l]], g2 = d_iq3xxs_grid[qs[8 * sub + 2 * l + 1]];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                y[8 * l + j] = db * (float)(uint8_t)(g1 >> (8 * j)) * ((signs >> j) & 1 ? -1.0f : 1.0f);
                y[8 * l + 4 + j] = db * (float)(uint8_t)(g2 >> (8 * j)) * ((signs >> (j + 4)) & 1 ? -1.0f : 1.0f);
            }
        }
        break;
    }
    case SHC_TYPE_IQ3_S: {
        const float d = ldh(blk);
        const uint8_t *qs = blk + 2, *qh = blk + 66, *sg = blk + 74, *sc = blk + 106;
        const float db = (sub % 2 == 0) ? d * (float)(1 + 2 * (sc[sub / 2] & 0xF)) : d * (float)(1 + 2 * (sc[sub / 2] >> 4));
#pragma unroll
        for (int l = 0; l < 4; l++) {
            const int i1 = qs[8 * sub + 2 * l] | ((qh[sub] << (8 - 2 * l)) & 256);
            const int i2 = qs[8 * sub + 2 * l + 1] | ((qh[sub] << (7 - 2 * l)) & 256);
            const uint32_t g1 = d_iq3s_grid[i1], g2 = d_iq3s_grid[i2];
            const uint8_t s = sg[4 * sub + l];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                y[8 * l + j] = db * (float)(uint8_t)(g1 >> (8 * j)) * ((s >> j) & 1 ? -1.0f : 1.0f);
                y[8 * l + 4 + j] = db * (float)(uint8_t)(g2 >> (8 * j)) * ((s >> (j + 4)) & 1 ? -1.0f : 1.0f);
            }
        }
        break;
    }
    case SHC_TYPE_IQ4_NL: {
        const float d = ldh(blk);
        const uint8_t *qs = blk + 2;
#pragma unroll
        for (int j = 0; j < 16; j++) {
            y[j] = d * (float)d_kvalues_iq4nl[qs[j] & 0xF];
            y[16 + j] = d * (float)d_kvalues_iq4nl[qs[j] >> 4];
        }
        break;
    }
    case SHC_TYPE_IQ4_XS: {
        const float d = ldh(blk);
        const uint16_t sh = (uint16_t)(blk[2] | (blk[3] << 8));
        const uint8_t *sl = blk + 4, *qs = blk + 8 + 16 * sub;
        const int ls = ((sl[sub / 2] >> (4 * (sub % 2))) & 0xF) | (((sh >> (2 * sub)) & 3) << 4);
        const float dl = d * (float)(ls - 32);
#pragma unroll
        for (int j = 0; j < 16; j++) {
            y[j] = dl * (float)d_kvalues_iq4nl[qs[j] & 0xF];
            y[16 + j] = dl * (float)d_kvalues_iq4nl[qs[j] >> 4];
        }
        break;
    }
    default:
        break;
    }
}

// Elementwise "encodings" (quant.rs:546-560) round-tripped to f32.
__device__ __forceinline__ float roundtrip_plain(uint32_t type, float x) {
    if (type == SHC_TYPE_F16) return f16_val(f16_bits(x));
    if (type == SHC_TYPE_BF16) return __uint_as_float(__float_as_uint(x) & 0xFFFF0000u);
    return x;
}

}  // namespace shc
