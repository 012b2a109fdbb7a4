/* CPU oracle for the shoehorn quantization hot path — TEST INFRASTRUCTURE.
 *
 * A strict-IEEE C restatement of the reference's Rust encoders and decoders,
 * function by function, keeping every operand order of the reference so that
 * the f32 roundings are the same:
 *   src/quant.rs      make_qx_quants 34-73, make_qkx3_quants 77-141,
 *                     element_weights 144-151, row_sigma2 153-155,
 *                     enc_q8_0 159-169, enc_q4_0 171-181, enc_q5_0 183-198,
 *                     enc_q4_1 200-211, enc_q5_1 213-229, enc_q6_k 231-291,
 *                     enc_qk45 294-379, decoders 383-537, encode_row 543-578,
 *                     decode_row 581-615, row_error 618-630
 *   src/quant_iq.rs   build_grid 44-96, expand_kgrid 100-112, grids 114-133,
 *                     find_best_neighbour 137-167, make_qp_quants 170-241,
 *                     signs_with_parity 245-271, enc_iq2_xxs 275-407,
 *                     enc_iq2_xs 430-563, enc_iq2_s 589-730, enc_iq3 758-935,
 *                     best_index_int8 1002-1024, iq4_impl 1027-1135,
 *                     decoders 409-426, 565-585, 732-754, 944-998, 1159-1189
 *   src/main.rs       encode_tensor 663-686, measuring closure 549-563
 *   src/imatrix.rs    row_slice 124-141
 *
 * Rust semantics reproduced here:
 *   - f32::round is round-half-away-from-zero (roundf), `as i32` saturates
 *     and maps NaN to 0 (nearest_int below);
 *   - half 2.7.1 f16::from_f32 is IEEE binary16 round-to-nearest-even;
 *   - f32::max / f32::min ignore NaN; for +0/-0 this file follows the
 *     aarch64 FMAXNM/FMINNM result (-0 < +0), the platform the reference's
 *     published numbers were produced on;
 *   - no FMA contraction (build with -ffp-contract=off).
 *
 * Parity status: the reference's own tests pin sizes, tolerances and grid
 * structure only; no byte-level golden vector exists and the Rust toolchain
 * is absent, so byte parity with the Rust binary is not pinned directly.
 */
#include "shoehorn_oracle.h"

#include <math.h>
#include <pthread.h>
#ifndef SH_OPCOUNT
#include <stdatomic.h>
#endif
#include <stdlib.h>
#include <string.h>

#include "iq_tables.h"

/* ---------------- ggml type ids (gguf.rs:36-83) ---------------- */
enum {
    T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q4_1 = 3, T_Q5_0 = 6, T_Q5_1 = 7, T_Q8_0 = 8,
    T_Q2_K = 10, T_Q3_K = 11, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14, T_IQ2_XXS = 16, T_IQ2_XS = 17, T_IQ3_XXS = 18,
    T_IQ4_NL = 20, T_IQ3_S = 21, T_IQ2_S = 22, T_IQ4_XS = 23, T_BF16 = 30
};

static const uint8_t kmask_iq2xs[8] = SH_KMASK_IQ2XS_DATA;
static const uint8_t ksigns_iq2xs[128] = SH_KSIGNS_IQ2XS_DATA;
static const uint64_t iq2xxs_grid[256] = SH_IQ2XXS_GRID_DATA;
static const uint64_t iq2xs_grid[512] = SH_IQ2XS_GRID_DATA;
static const uint64_t iq2s_grid[1024] = SH_IQ2S_GRID_DATA;
static const uint32_t iq3xxs_grid[256] = SH_IQ3XXS_GRID_DATA;
static const uint32_t iq3s_grid[512] = SH_IQ3S_GRID_DATA;
static const int8_t kvalues_iq4nl[16] = SH_KVALUES_IQ4NL_DATA;
static const uint16_t kgrid_2bit_256[256] = SH_KGRID_2BIT_256_DATA;
static const uint16_t kgrid_2bit_512[512] = SH_KGRID_2BIT_512_DATA;
static const uint16_t kgrid_2bit_1024[1024] = SH_KGRID_2BIT_1024_DATA;
static const uint16_t kgrid_256[256] = SH_KGRID_256_DATA;
static const uint16_t kgrid_512[512] = SH_KGRID_512_DATA;

/* gguf.rs:86-107 block_layout */
static int block_layout(uint32_t t, int64_t *bs, int64_t *tb) {
    switch (t) {
    case T_F32: *bs = 1; *tb = 4; return 1;
    case T_F16: case T_BF16: *bs = 1; *tb = 2; return 1;
    case T_Q4_0: *bs = 32; *tb = 18; return 1;
    case T_Q4_1: *bs = 32; *tb = 20; return 1;
    case T_Q5_0: *bs = 32; *tb = 22; return 1;
    case T_Q5_1: *bs = 32; *tb = 24; return 1;
    case T_Q8_0: *bs = 32; *tb = 34; return 1;
    case T_Q2_K: *bs = 256; *tb = 84; return 1;
    case T_Q3_K: *bs = 256; *tb = 110; return 1;
    case T_Q4_K: *bs = 256; *tb = 144; return 1;
    case T_Q5_K: *bs = 256; *tb = 176; return 1;
    case T_Q6_K: *bs = 256; *tb = 210; return 1;
    case T_IQ2_XXS: *bs = 256; *tb = 66; return 1;
    case T_IQ2_XS: *bs = 256; *tb = 74; return 1;
    case T_IQ2_S: *bs = 256; *tb = 82; return 1;
    case T_IQ3_XXS: *bs = 256; *tb = 98; return 1;
    case T_IQ3_S: *bs = 256; *tb = 110; return 1;
    case T_IQ4_NL: *bs = 32; *tb = 18; return 1;
    case T_IQ4_XS: *bs = 256; *tb = 136; return 1;
    default: return 0;
    }
}

int64_t oq_row_bytes(uint32_t type, int64_t n) {
    int64_t bs, tb;
    if (!block_layout(type, &bs, &tb) || n < 0 || n % bs != 0) return -1;
    return n / bs * tb;
}

/* ---------------- scalar semantics ---------------- */

/* The op-counting build (opcount/) supplies counted copies of nearest_int,
 * rmaxf and rminf with the same semantics. */
#ifndef SH_OPCOUNT
/* quant.rs:16 nearest_int: f32::round (half away from zero), `as i32`. */
int32_t oq_nearest_int(float x) {
    float r = roundf(x);
    if (r != r) return 0;
    if (r >= 2147483648.0f) return INT32_MAX;
    if (r <= -2147483648.0f) return INT32_MIN;
    return (int32_t)r;
}
#endif
#define nearest_int oq_nearest_int

static inline int32_t clampi(int32_t v, int32_t lo, int32_t hi) { return v < lo ? lo : (v > hi ? hi : v); }
static inline int32_t mini(int32_t a, int32_t b) { return a < b ? a : b; }

#ifndef SH_OPCOUNT
/* f32::max / f32::min: NaN-ignoring; -0 < +0. */
static inline float rmaxf(float a, float b) {
    if (a != a) return b;
    if (b != b) return a;
    if (a > b) return a;
    if (b > a) return b;
    return signbit(a) ? b : a;
}
static inline float rminf(float a, float b) {
    if (a != a) return b;
    if (b != b) return a;
    if (a < b) return a;
    if (b < a) return b;
    return signbit(a) ? a : b;
}
#endif

/* IEEE binary16, round to nearest even (half::f16::from_f32). */
uint16_t oq_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xFFu;
    uint32_t man = x & 0x7FFFFFu;
    if (exp == 0xFFu) {
        if (man == 0) return (uint16_t)(sign | 0x7C00u);
        return (uint16_t)(sign | 0x7E00u | (man >> 13));
    }
    int32_t e = (int32_t)exp - 127 + 15;
    if (e >= 0x1F) return (uint16_t)(sign | 0x7C00u);
    if (e <= 0) {
        /* subnormal or zero in f16: value = man24 * 2^(exp-150); f16 unit 2^-24 */
        if (e < -10) return (uint16_t)sign; /* below half of the smallest subnormal */
        uint32_t m = man | 0x800000u;
        uint32_t shift = (uint32_t)(14 - e); /* 24-bit mantissa -> units of 2^-24 */
        uint32_t q = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t q = ((uint32_t)e << 10) | (man >> 13);
    uint32_t rem = man & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++; /* carry may reach inf: correct */
    return (uint16_t)(sign | q);
}

float oq_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    uint32_t x;
    if (exp == 0) {
        if (man == 0) {
            x = sign;
        } else {
            int e = -1;
            do { man <<= 1; e++; } while (!(man & 0x400u));
            man &= 0x3FFu;
            x = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 0x1F) {
        x = sign | 0x7F800000u | (man << 13);
    } else {
        x = sign | ((exp - 15 + 127) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

static inline void put_f16(uint8_t *p, float v) {
    uint16_t h = oq_f32_to_f16(v);
    p[0] = (uint8_t)(h & 0xFF);
    p[1] = (uint8_t)(h >> 8);
}
static inline float get_f16(const uint8_t *p) { return oq_f16_to_f32((uint16_t)(p[0] | (p[1] << 8))); }
static inline uint32_t rd_u32(const uint8_t *p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
static inline void wr_u32(uint8_t *p, uint32_t v) {
    p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); p[2] = (uint8_t)(v >> 16); p[3] = (uint8_t)(v >> 24);
}

#define GROUP_MAX_EPS 1e-15f
#define GROUP_MAX_EPS_IQ3_XXS 1e-8f
#define GROUP_MAX_EPS_IQ2_S 1e-8f

/* ---------------- quant.rs search routines ---------------- */

/* quant.rs:34-73 */
static float make_qx_quants(const float *x, int n, int nmax, const float *w, uint8_t *ls) {
    float max = 0.0f, amax = 0.0f;
    for (int i = 0; i < n; i++) {
        float a = fabsf(x[i]);
        if (a > amax) { amax = a; max = x[i]; }
    }
    if (amax < GROUP_MAX_EPS) {
        memset(ls, nmax, (size_t)n);
        return 0.0f;
    }
    float best_scale = 0.0f, best = 0.0f;
    int first = 1;
    uint8_t cand[32];
    for (int is = -9; is <= 9; is++) {
        float iscale = -((float)nmax + 0.1f * (float)is) / max;
        float sumlx = 0.0f, suml2 = 0.0f;
        for (int i = 0; i < n; i++) {
            int32_t l = clampi(nearest_int(iscale * x[i]), -nmax, nmax - 1);
            cand[i] = (uint8_t)(l + nmax);
            float wi = w[i];
            sumlx += wi * x[i] * (float)l;
            suml2 += wi * (float)(l * l);
        }
        if (suml2 > 0.0f && (first || sumlx * sumlx > best * suml2)) {
            float scale = sumlx / suml2;
            best_scale = scale;
            best = scale * sumlx;
            memcpy(ls, cand, (size_t)n);
            first = 0;
        }
    }
    return best_scale;
}

/* quant.rs:77-141 ; returns (scale, min) */
static void make_qkx3_quants(const float *x, int n, int nmax, const float *w, uint8_t *ls, float rmin,
                             float rdelta, int nstep, float *out_scale, float *out_min) {
    float vmin = INFINITY, vmax = -INFINITY;
    for (int i = 0; i < n; i++) vmin = rminf(vmin, x[i]);
    vmin = rminf(vmin, 0.0f);
    for (int i = 0; i < n; i++) vmax = rmaxf(vmax, x[i]);
    if (vmax <= vmin) {
        memset(ls, 0, (size_t)n);
        *out_scale = 0.0f;
        *out_min = vmin;
        return;
    }
    float iscale = (float)nmax / (vmax - vmin);
    float scale = 1.0f / iscale;
    float best_err = 0.0f;
    for (int i = 0; i < n; i++) {
        int32_t l = clampi(nearest_int(iscale * (x[i] - vmin)), 0, nmax);
        ls[i] = (uint8_t)l;
        float diff = scale * (float)l + vmin - x[i];
        best_err += w[i] * diff * diff;
    }
    float best_min = vmin;
    uint8_t laux[32];
    for (int is = 0; is <= nstep; is++) {
        iscale = (rmin + rdelta * (float)is + (float)nmax) / (vmax - vmin);
        float sum_w = 0.0f, sum_x = 0.0f, sum_l = 0.0f, sum_l2 = 0.0f, sum_xl = 0.0f;
        for (int i = 0; i < n; i++) {
            int32_t l = clampi(nearest_int(iscale * (x[i] - vmin)), 0, nmax);
            laux[i] = (uint8_t)l;
            float wi = w[i];
            sum_w += wi;
            sum_x += wi * x[i];
            sum_l += wi * (float)l;
            sum_l2 += wi * (float)(l * l);
            sum_xl += wi * (float)l * x[i];
        }
        float d = sum_w * sum_l2 - sum_l * sum_l;
        if (d > 0.0f) {
            float this_scale = (sum_w * sum_xl - sum_x * sum_l) / d;
            float this_min = (sum_l2 * sum_x - sum_l * sum_xl) / d;
            if (this_min > 0.0f) {
                this_min = 0.0f;
                this_scale = sum_l2 > 0.0f ? sum_xl / sum_l2 : 0.0f;
            }
            float err = 0.0f;
            for (int i = 0; i < n; i++) {
                float diff = this_scale * (float)laux[i] + this_min - x[i];
                err += w[i] * diff * diff;
            }
            if (err < best_err) {
                best_err = err;
                scale = this_scale;
                best_min = this_min;
                memcpy(ls, laux, (size_t)n);
            }
        }
    }
    *out_scale = scale;
    *out_min = best_min;
}

/* quant.rs:144-151 */
static void element_weights(const float *x, int n, const float *im, float sigma2, float *w) {
    for (int i = 0; i < n; i++) {
        float base = im ? im[i] : 1.0f;
        w[i] = base * sqrtf(sigma2 + x[i] * x[i]);
    }
}

/* quant.rs:153-155: sequential f32 fold over the whole row. */
static float row_sigma2(const float *x, int64_t n) {
    float s = 0.0f;
    for (int64_t i = 0; i < n; i++) s += x[i] * x[i];
    return s / (float)n;
}

/* ---------------- quant.rs encoders ---------------- */

/* quant.rs:159-169 */
static void enc_q8_0(const float *x, int64_t n, uint8_t *out) {
    for (int64_t b = 0; b < n / 32; b++) {
        const float *blk = x + 32 * b;
        uint8_t *o = out + 34 * b;
        float amax = 0.0f;
        for (int j = 0; j < 32; j++) amax = rmaxf(amax, fabsf(blk[j]));
        float d = amax / 127.0f;
        float id = d > 0.0f ? 1.0f / d : 0.0f;
        put_f16(o, d);
        for (int j = 0; j < 32; j++) o[2 + j] = (uint8_t)(int8_t)clampi(nearest_int(blk[j] * id), -127, 127);
    }
}

/* quant.rs:171-181 */
static void enc_q4_0(const float *x, int64_t n, const float *im, float sigma2, uint8_t *out) {
    /* one level vector for the whole row, as the reference's `ls` outlives the
       block loop: a block where no grid is accepted keeps the previous levels */
    uint8_t ls[32] = {0};
    float w[32];
    for (int64_t b = 0; b < n / 32; b++) {
        const float *blk = x + 32 * b;
        uint8_t *o = out + 18 * b;
        element_weights(blk, 32, im ? im + 32 * b : NULL, sigma2, w);
        float d = make_qx_quants(blk, 32, 8, w, ls);
        put_f16(o, d);
        for (int j = 0; j < 16; j++) o[2 + j] = (uint8_t)((ls[j] & 0xF) | (ls[j + 16] << 4));
    }
}

/* quant.rs:183-198 */
static void enc_q5_0(const float *x, int64_t n, const float *im, float sigma2, uint8_t *out) {
    uint8_t ls[32] = {0};
    float w[32];
    for (int64_t b = 0; b < n / 32; b++) {
        const float *blk = x + 32 * b;
        uint8_t *o = out + 22 * b;
        element_weights(blk, 32, im ? im + 32 * b : NULL, sigma2, w);
        float d = make_qx_quants(blk, 32, 16, w, ls);
        put_f16(o, d);
        uint32_t qh = 0;
        for (int j = 0; j < 32; j++) qh |= ((uint32_t)((ls[j] >> 4) & 1)) << j;
        wr_u32(o + 2, qh);
        for (int j = 0; j < 16; j++) o[6 + j] = (uint8_t)((ls[j] & 0xF) | ((ls[j + 16] & 0xF) << 4));
    }
}

/* quant.rs:200-211 */
static void enc_q4_1(const float *x, int64_t n, const float *im, float sigma2, uint8_t *out) {
    uint8_t ls[32] = {0};
    float w[32];
    for (int64_t b = 0; b < n / 32; b++) {
        const float *blk = x + 32 * b;
        uint8_t *o = out + 20 * b;
        element_weights(blk, 32, im ? im + 32 * b : NULL, sigma2, w);
        float d, mn;
        make_qkx3_quants(blk, 32, 15, w, ls, -0.9f, 0.05f, 36, &d, &mn);
        put_f16(o, d);
        put_f16(o + 2, mn);
        for (int j = 0; j < 16; j++) o[4 + j] = (uint8_t)((ls[j] & 0xF) | (ls[j + 16] << 4));
    }
}

/* quant.rs:213-229 */
static void enc_q5_1(const float *x, int64_t n, const float *im, float sigma2, uint8_t *out) {
    uint8_t ls[32] = {0};
    float w[32];
    for (int64_t b = 0; b < n / 32; b++) {
        const float *blk = x + 32 * b;
        uint8_t *o = out + 24 * b;
        element_weights(blk, 32, im ? im + 32 * b : NULL, sigma2, w);
        float d, mn;
        make_qkx3_quants(blk, 32, 31, w, ls, -0.9f, 0.05f, 36, &d, &mn);
        put_f16(o, d);
        put_f16(o + 2, mn);
        uint32_t qh = 0;
        for (int j = 0; j < 32; j++) qh |= ((uint32_t)((ls[j] >> 4) & 1)) << j;
        wr_u32(o + 4, qh);
        for (int j = 0; j < 16; j++) o[8 + j] = (uint8_t)((ls[j] & 0xF) | ((ls[j + 16] & 0xF) << 4));
    }
}

/* quant.rs:231-291 */
static void enc_q6_k(const float *x, int64_t n, const float *im, float sigma2, uint8_t *out) {
    uint8_t l_all[256];
    float w[16];
    for (int64_t bi = 0; bi < n / 256; bi++) {
        const float *blk = x + 256 * bi;
        uint8_t *o = out + 210 * bi;
        float scales[16];
        float max_abs_scale = 0.0f, max_scale = 0.0f;
        for (int sb = 0; sb < 16; sb++) {
            const float *xs = blk + sb * 16;
            element_weights(xs, 16, im ? im + bi * 256 + sb * 16 : NULL, sigma2, w);
            uint8_t ls[16];
            float s = make_qx_quants(xs, 16, 32, w, ls);
            scales[sb] = s;
            if (fabsf(s) > max_abs_scale) { max_abs_scale = fabsf(s); max_scale = s; }
        }
        memset(o, 0, 210);
        if (max_abs_scale < GROUP_MAX_EPS) continue;
        float iscale = -128.0f / max_scale;
        float d = 1.0f / iscale;
        int8_t qscales[16];
        for (int sb = 0; sb < 16; sb++) qscales[sb] = (int8_t)(uint8_t)(mini(nearest_int(iscale * scales[sb]), 127) & 0xFF);
        for (int sb = 0; sb < 16; sb++) {
            float dd = d * (float)qscales[sb];
            if (dd == 0.0f) {
                for (int j = 0; j < 16; j++) l_all[sb * 16 + j] = 32;
                continue;
            }
            for (int j = 0; j < 16; j++) {
                int32_t l = clampi(nearest_int(blk[sb * 16 + j] / dd), -32, 31);
                l_all[sb * 16 + j] = (uint8_t)(l + 32);
            }
        }
        for (int h = 0; h < 2; h++) {
            const uint8_t *lo = l_all + h * 128;
            uint8_t *ql = o + h * 64;
            uint8_t *qh = o + 128 + h * 32;
            for (int l = 0; l < 32; l++) {
                ql[l] = (uint8_t)((lo[l] & 0xF) | ((lo[l + 64] & 0xF) << 4));
                ql[32 + l] = (uint8_t)((lo[l + 32] & 0xF) | ((lo[l + 96] & 0xF) << 4));
                qh[l] = (uint8_t)((lo[l] >> 4) | ((lo[l + 32] >> 4) << 2) | ((lo[l + 64] >> 4) << 4) | ((lo[l + 96] >> 4) << 6));
            }
        }
        for (int sb = 0; sb < 16; sb++) o[192 + sb] = (uint8_t)qscales[sb];
        put_f16(o + 208, d);
    }
}

/* quant.rs:294-379 (nmax 15: Q4_K, 31: Q5_K) */
static void enc_qk45(const float *x, int64_t n, const float *im, float sigma2, int nmax, uint8_t *out) {
    int five = nmax == 31;
    int64_t block_bytes = five ? 176 : 144;
    uint8_t l_all[256];
    float w[32];
    for (int64_t bi = 0; bi < n / 256; bi++) {
        const float *blk = x + 256 * bi;
        uint8_t *o = out + block_bytes * bi;
        float scales[8], mins[8];
        for (int sb = 0; sb < 8; sb++) {
            const float *xs = blk + sb * 32;
            element_weights(xs, 32, im ? im + bi * 256 + sb * 32 : NULL, sigma2, w);
            uint8_t ls[32];
            float s, mn;
            make_qkx3_quants(xs, 32, nmax, w, ls, -0.9f, 0.05f, 36, &s, &mn);
            scales[sb] = s;
            mins[sb] = -mn;
        }
        float max_scale = 0.0f, max_min = 0.0f;
        for (int sb = 0; sb < 8; sb++) max_scale = rmaxf(max_scale, scales[sb]);
        for (int sb = 0; sb < 8; sb++) max_min = rmaxf(max_min, mins[sb]);
        float inv_scale = max_scale > 0.0f ? 63.0f / max_scale : 0.0f;
        float inv_min = max_min > 0.0f ? 63.0f / max_min : 0.0f;
        uint8_t sc[12] = {0};
        uint8_t lsq[8], lmq[8];
        for (int sb = 0; sb < 8; sb++) {
            lsq[sb] = (uint8_t)clampi(nearest_int(inv_scale * scales[sb]), 0, 63);
            lmq[sb] = (uint8_t)clampi(nearest_int(inv_min * mins[sb]), 0, 63);
            if (sb < 4) {
                sc[sb] = lsq[sb];
                sc[sb + 4] = lmq[sb];
            } else {
                sc[sb + 4] = (uint8_t)((lsq[sb] & 0xF) | ((lmq[sb] & 0xF) << 4));
                sc[sb - 4] |= (uint8_t)((lsq[sb] >> 4) << 6);
                sc[sb] |= (uint8_t)((lmq[sb] >> 4) << 6);
            }
        }
        float d = max_scale / 63.0f;
        float dmin = max_min / 63.0f;
        for (int sb = 0; sb < 8; sb++) {
            float dsub = d * (float)lsq[sb];
            float msub = dmin * (float)lmq[sb];
            if (dsub == 0.0f) {
                for (int j = 0; j < 32; j++) l_all[sb * 32 + j] = 0;
                continue;
            }
            for (int j = 0; j < 32; j++)
                l_all[sb * 32 + j] = (uint8_t)clampi(nearest_int((blk[sb * 32 + j] + msub) / dsub), 0, nmax);
        }
        memset(o, 0, (size_t)block_bytes);
        put_f16(o, d);
        put_f16(o + 2, dmin);
        memcpy(o + 4, sc, 12);
        if (five) {
            uint8_t *qh = o + 16, *qs = o + 48;
            for (int chunk = 0; chunk < 4; chunk++) {
                uint8_t u1 = (uint8_t)(1u << (chunk * 2)), u2 = (uint8_t)(2u << (chunk * 2));
                for (int l = 0; l < 32; l++) {
                    uint8_t a = l_all[chunk * 64 + l], b = l_all[chunk * 64 + 32 + l];
                    qs[chunk * 32 + l] = (uint8_t)((a & 0xF) | ((b & 0xF) << 4));
                    if (a >= 16) qh[l] |= u1;
                    if (b >= 16) qh[l] |= u2;
                }
            }
        } else {
            uint8_t *qs = o + 16;
            for (int chunk = 0; chunk < 4; chunk++)
                for (int l = 0; l < 32; l++)
                    qs[chunk * 32 + l] = (uint8_t)((l_all[chunk * 64 + l] & 0xF) | (l_all[chunk * 64 + 32 + l] << 4));
        }
    }
}

/* Q2_K and Q3_K.  The reference has no encoder for either type
 * (gguf.rs:13-34 lists no Q2_K/Q3_K), so these restate its own K-quant
 * recipes at 16-element sub-blocks, in the ggml block layouts that gguf-py
 * 0.19.0 decodes:
 *   Q2_K = enc_qk45 with make_qkx3_quants(n 16, nmax 3) and 4-bit scale/min
 *          codes (max/15), bytes scales[16] (scale | min << 4), qs[64], d, dmin;
 *   Q3_K = enc_q6_k with make_qx_quants(n 16, nmax 4) and 6-bit signed scale
 *          codes (iscale = -32/max), bytes hmask[32], qs[64], scales[12], d.
 * Element e of a super-block: qs byte (e/128)*32 + e%32 at bit 2*((e%128)/32);
 * Q3_K's high bit in hmask byte e%32, bit e/32. */
static void enc_q2_k(const float *x, int64_t n, const float *im, float sigma2, uint8_t *out) {
    uint8_t l_all[256];
    float w[16];
    for (int64_t bi = 0; bi < n / 256; bi++) {
        const float *blk = x + 256 * bi;
        uint8_t *o = out + 84 * bi;
        float scales[16], mins[16];
        for (int sb = 0; sb < 16; sb++) {
            const float *xs = blk + sb * 16;
            element_weights(xs, 16, im ? im + bi * 256 + sb * 16 : NULL, sigma2, w);
            uint8_t ls[16];
            float sc, mn;
            make_qkx3_quants(xs, 16, 3, w, ls, -0.9f, 0.05f, 36, &sc, &mn);
            scales[sb] = sc;
            mins[sb] = -mn;
        }
        float max_scale = 0.0f, max_min = 0.0f;
        for (int sb = 0; sb < 16; sb++) max_scale = rmaxf(max_scale, scales[sb]);
        for (int sb = 0; sb < 16; sb++) max_min = rmaxf(max_min, mins[sb]);
        float inv_scale = max_scale > 0.0f ? 15.0f / max_scale : 0.0f;
        float inv_min = max_min > 0.0f ? 15.0f / max_min : 0.0f;
        float d = max_scale / 15.0f;
        float dmin = max_min / 15.0f;
        memset(o, 0, 84);
        for (int sb = 0; sb < 16; sb++) {
            int32_t lsq = clampi(nearest_int(inv_scale * scales[sb]), 0, 15);
            int32_t lmq = clampi(nearest_int(inv_min * mins[sb]), 0, 15);
            o[sb] = (uint8_t)(lsq | (lmq << 4));
            float dsub = d * (float)lsq;
            float msub = dmin * (float)lmq;
            for (int j = 0; j < 16; j++)
                l_all[sb * 16 + j] = dsub == 0.0f ? 0 : (uint8_t)clampi(nearest_int((blk[sb * 16 + j] + msub) / dsub), 0, 3);
        }
        for (int e = 0; e < 256; e++) o[16 + (e / 128) * 32 + e % 32] |= (uint8_t)(l_all[e] << (2 * ((e % 128) / 32)));
        put_f16(o + 80, d);
        put_f16(o + 82, dmin);
    }
}
static void enc_q3_k(const float *x, int64_t n, const float *im, float sigma2, uint8_t *out) {
    uint8_t l_all[256];
    float w[16];
    for (int64_t bi = 0; bi < n / 256; bi++) {
        const float *blk = x + 256 * bi;
        uint8_t *o = out + 110 * bi;
        float scales[16];
        float max_abs_scale = 0.0f, max_scale = 0.0f;
        for (int sb = 0; sb < 16; sb++) {
            const float *xs = blk + sb * 16;
            element_weights(xs, 16, im ? im + bi * 256 + sb * 16 : NULL, sigma2, w);
            uint8_t ls[16];
            float sc = make_qx_quants(xs, 16, 4, w, ls);
            scales[sb] = sc;
            if (fabsf(sc) > max_abs_scale) { max_abs_scale = fabsf(sc); max_scale = sc; }
        }
        memset(o, 0, 110);
        if (max_abs_scale < GROUP_MAX_EPS) continue;
        float iscale = -32.0f / max_scale;
        float d = 1.0f / iscale;
        for (int sb = 0; sb < 16; sb++) {
            int32_t q = clampi(nearest_int(iscale * scales[sb]), -32, 31);
            uint32_t u = (uint32_t)(q + 32);
            o[96 + sb % 8] |= (uint8_t)((u & 0xF) << (4 * (sb / 8)));
            o[96 + 8 + sb % 4] |= (uint8_t)((u >> 4) << (2 * (sb / 4)));
            float dd = d * (float)q;
            for (int j = 0; j < 16; j++)
                l_all[sb * 16 + j] = dd == 0.0f ? 4 : (uint8_t)(clampi(nearest_int(blk[sb * 16 + j] / dd), -4, 3) + 4);
        }
        for (int e = 0; e < 256; e++) {
            o[32 + (e / 128) * 32 + e % 32] |= (uint8_t)((l_all[e] & 3) << (2 * ((e % 128) / 32)));
            if (l_all[e] & 4) o[e % 32] |= (uint8_t)(1u << (e / 32));
        }
        put_f16(o + 108, d);
    }
}

/* ---------------- quant.rs decoders ---------------- */

static void dec_q8_0(const uint8_t *data, int64_t n, float *out) {
    for (int64_t b = 0; b < n / 32; b++) {
        const uint8_t *blk = data + 34 * b;
        float d = get_f16(blk);
        for (int j = 0; j < 32; j++) out[32 * b + j] = d * (float)(int8_t)blk[2 + j];
    }
}
static void dec_q4_0(const uint8_t *data, int64_t n, float *out) {
    for (int64_t b = 0; b < n / 32; b++) {
        const uint8_t *blk = data + 18 * b;
        float d = get_f16(blk);
        const uint8_t *qs = blk + 2;
        for (int h = 0; h < 2; h++)
            for (int j = 0; j < 16; j++) {
                int q = h == 0 ? (qs[j] & 0xF) : (qs[j] >> 4);
                out[32 * b + h * 16 + j] = d * (float)(q - 8);
            }
    }
}
static void dec_q5_0(const uint8_t *data, int64_t n, float *out) {
    for (int64_t b = 0; b < n / 32; b++) {
        const uint8_t *blk = data + 22 * b;
        float d = get_f16(blk);
        uint32_t qh = rd_u32(blk + 2);
        const uint8_t *qs = blk + 6;
        for (int h = 0; h < 2; h++)
            for (int j = 0; j < 16; j++) {
                int idx = h * 16 + j;
                uint32_t lo = h == 0 ? (qs[j] & 0xFu) : (uint32_t)(qs[j] >> 4);
                uint32_t q = lo | (((qh >> idx) & 1u) << 4);
                out[32 * b + idx] = d * (float)((int32_t)q - 16);
            }
    }
}
static void dec_q4_1(const uint8_t *data, int64_t n, float *out) {
    for (int64_t b = 0; b < n / 32; b++) {
        const uint8_t *blk = data + 20 * b;
        float d = get_f16(blk), m = get_f16(blk + 2);
        const uint8_t *qs = blk + 4;
        for (int h = 0; h < 2; h++)
            for (int j = 0; j < 16; j++) {
                int q = h == 0 ? (qs[j] & 0xF) : (qs[j] >> 4);
                out[32 * b + h * 16 + j] = d * (float)q + m;
            }
    }
}
static void dec_q5_1(const uint8_t *data, int64_t n, float *out) {
    for (int64_t b = 0; b < n / 32; b++) {
        const uint8_t *blk = data + 24 * b;
        float d = get_f16(blk), m = get_f16(blk + 2);
        uint32_t qh = rd_u32(blk + 4);
        const uint8_t *qs = blk + 8;
        for (int h = 0; h < 2; h++)
            for (int j = 0; j < 16; j++) {
                int idx = h * 16 + j;
                uint32_t lo = h == 0 ? (qs[j] & 0xFu) : (uint32_t)(qs[j] >> 4);
                uint32_t q = lo | (((qh >> idx) & 1u) << 4);
                out[32 * b + idx] = d * (float)q + m;
            }
    }
}
static void dec_q6_k(const uint8_t *data, int64_t n, float *out) {
    for (int64_t b = 0; b < n / 256; b++) {
        const uint8_t *blk = data + 210 * b;
        float d = get_f16(blk + 208);
        float *y = out + 256 * b;
        for (int h = 0; h < 2; h++) {
            const uint8_t *ql = blk + h * 64, *qh = blk + 128 + h * 32;
            const int8_t *sc = (const int8_t *)(blk + 192 + h * 8);
            for (int l = 0; l < 32; l++) {
                int is = l / 16;
                int q1 = ((ql[l] & 0xF) | ((qh[l] & 3) << 4)) - 32;
                int q2 = ((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                int q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                int q4 = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                int o = h * 128;
                y[o + l] = d * (float)sc[is] * (float)q1;
                y[o + l + 32] = d * (float)sc[is + 2] * (float)q2;
                y[o + l + 64] = d * (float)sc[is + 4] * (float)q3;
                y[o + l + 96] = d * (float)sc[is + 6] * (float)q4;
            }
        }
    }
}
static void dec_q2_k(const uint8_t *data, int64_t n, float *out) {
    for (int64_t bi = 0; bi < n / 256; bi++) {
        const uint8_t *b = data + 84 * bi;
        const float d = get_f16(b + 80), dmin = get_f16(b + 82);
        for (int e = 0; e < 256; e++) {
            const uint8_t sc = b[e / 16];
            const int q = (b[16 + (e / 128) * 32 + e % 32] >> (2 * ((e % 128) / 32))) & 3;
            out[256 * bi + e] = (d * (float)(sc & 0xF)) * (float)q - dmin * (float)(sc >> 4);
        }
    }
}
static void dec_q3_k(const uint8_t *data, int64_t n, float *out) {
    for (int64_t bi = 0; bi < n / 256; bi++) {
        const uint8_t *b = data + 110 * bi;
        const float d = get_f16(b + 108);
        for (int e = 0; e < 256; e++) {
            const int sb = e / 16;
            const int u = ((b[96 + sb % 8] >> (4 * (sb / 8))) & 0xF) | (((b[104 + sb % 4] >> (2 * (sb / 4))) & 3) << 4);
            const int lo = (b[32 + (e / 128) * 32 + e % 32] >> (2 * ((e % 128) / 32))) & 3;
            const int hi = (b[e % 32] >> (e / 32)) & 1;
            out[256 * bi + e] = (d * (float)(u - 32)) * (float)(lo - (hi ? 0 : 4));
        }
    }
}
/* quant.rs:477-486 */
static void get_scale_min_k4(int j, const uint8_t *q, uint8_t *sc, uint8_t *m) {
    if (j < 4) {
        *sc = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *sc = (uint8_t)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
        *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}
static void dec_q4_k(const uint8_t *data, int64_t n, float *out) {
    for (int64_t b = 0; b < n / 256; b++) {
        const uint8_t *blk = data + 144 * b;
        float d = get_f16(blk), dmin = get_f16(blk + 2);
        const uint8_t *scales = blk + 4, *qs = blk + 16;
        float *y = out + 256 * b;
        for (int chunk = 0; chunk < 4; chunk++) {
            uint8_t sc1, m1, sc2, m2;
            get_scale_min_k4(chunk * 2, scales, &sc1, &m1);
            get_scale_min_k4(chunk * 2 + 1, scales, &sc2, &m2);
            float d1 = d * (float)sc1, mm1 = dmin * (float)m1;
            float d2 = d * (float)sc2, mm2 = dmin * (float)m2;
            for (int l = 0; l < 32; l++) y[chunk * 64 + l] = d1 * (float)(qs[chunk * 32 + l] & 0xF) - mm1;
            for (int l = 0; l < 32; l++) y[chunk * 64 + 32 + l] = d2 * (float)(qs[chunk * 32 + l] >> 4) - mm2;
        }
    }
}
static void dec_q5_k(const uint8_t *data, int64_t n, float *out) {
    for (int64_t b = 0; b < n / 256; b++) {
        const uint8_t *blk = data + 176 * b;
        float d = get_f16(blk), dmin = get_f16(blk + 2);
        const uint8_t *scales = blk + 4, *qh = blk + 16, *qs = blk + 48;
        float *y = out + 256 * b;
        for (int chunk = 0; chunk < 4; chunk++) {
            uint8_t sc1, m1, sc2, m2;
            get_scale_min_k4(chunk * 2, scales, &sc1, &m1);
            get_scale_min_k4(chunk * 2 + 1, scales, &sc2, &m2);
            float d1 = d * (float)sc1, mm1 = dmin * (float)m1;
            float d2 = d * (float)sc2, mm2 = dmin * (float)m2;
            uint8_t u1 = (uint8_t)(1u << (chunk * 2)), u2 = (uint8_t)(2u << (chunk * 2));
            for (int l = 0; l < 32; l++) {
                float q = (float)(qs[chunk * 32 + l] & 0xF) + ((qh[l] & u1) ? 16.0f : 0.0f);
                y[chunk * 64 + l] = d1 * q - mm1;
            }
            for (int l = 0; l < 32; l++) {
                float q = (float)(qs[chunk * 32 + l] >> 4) + ((qh[l] & u2) ? 16.0f : 0.0f);
                y[chunk * 64 + 32 + l] = d2 * q - mm2;
            }
        }
    }
}

/* ---------------- quant_iq.rs: lattice structures ---------------- */

typedef struct {
    int8_t (*grid)[8];
    int grid_size, dim;
    int32_t *map;
    int kmap_size;
    uint16_t *neighbours;
    int64_t n_neighbours;
} grid_data;

typedef struct { int32_t d2; uint16_t j; } d2j;
static int cmp_d2j(const void *a, const void *b) {
    const d2j *x = (const d2j *)a, *y = (const d2j *)b;
    if (x->d2 != y->d2) return x->d2 < y->d2 ? -1 : 1;
    return (int)x->j - (int)y->j;
}

/* quant_iq.rs:100-112 */
static int8_t (*expand_kgrid(const uint16_t *packed, int n, int dim, int bits))[8] {
    int8_t (*p)[8] = calloc((size_t)n, 8);
    for (int i = 0; i < n; i++)
        for (int k = 0; k < dim; k++) p[i][k] = (int8_t)(2 * ((packed[i] >> (bits * k)) & ((1 << bits) - 1)) + 1);
    return p;
}

/* quant_iq.rs:44-96 */
static void build_grid(grid_data *g, int8_t (*points)[8], int grid_size, int dim, int kmap_size, int bits, int nwant) {
    g->grid = points;
    g->grid_size = grid_size;
    g->dim = dim;
    g->kmap_size = kmap_size;
    g->map = malloc(sizeof(int32_t) * (size_t)kmap_size);
    for (int i = 0; i < kmap_size; i++) g->map[i] = -1;
    for (int i = 0; i < grid_size; i++) {
        int index = 0;
        for (int k = 0; k < dim; k++) index |= ((points[i][k] - 1) / 2) << (bits * k);
        g->map[index] = i;
    }
    int64_t cap = 1 << 16, len = 0;
    uint16_t *nb = malloc(sizeof(uint16_t) * (size_t)cap);
    d2j *dist2 = malloc(sizeof(d2j) * (size_t)grid_size);
    for (int i = 0; i < kmap_size; i++) {
        if (g->map[i] >= 0) continue;
        int pos[8];
        for (int k = 0; k < dim; k++) pos[k] = 2 * ((i >> (bits * k)) & ((1 << bits) - 1)) + 1;
        for (int j = 0; j < grid_size; j++) {
            int d2 = 0;
            for (int k = 0; k < dim; k++) {
                int d = points[j][k] - pos[k];
                d2 += d * d;
            }
            dist2[j].d2 = d2;
            dist2[j].j = (uint16_t)j;
        }
        qsort(dist2, (size_t)grid_size, sizeof(d2j), cmp_d2j);
        if (len + grid_size + 1 > cap) {
            while (len + grid_size + 1 > cap) cap *= 2;
            nb = realloc(nb, sizeof(uint16_t) * (size_t)cap);
        }
        g->map[i] = -(int32_t)(len + 1);
        int64_t start = len;
        nb[len++] = 0;
        uint16_t cnt = 0;
        int nhave = 1;
        int d2 = dist2[0].d2;
        for (int t = 0; t < grid_size; t++) {
            if (dist2[t].d2 > d2) {
                if (nhave == nwant) break;
                d2 = dist2[t].d2;
                nhave++;
            }
            nb[len++] = dist2[t].j;
            cnt++;
        }
        nb[start] = cnt;
    }
    free(dist2);
    g->neighbours = nb;
    g->n_neighbours = len;
}

static grid_data G[5];
static pthread_once_t grid_once = PTHREAD_ONCE_INIT;
static void init_grids(void) {
    build_grid(&G[0], expand_kgrid(kgrid_2bit_256, 256, 8, 2), 256, 8, 43692, 2, 2);
    build_grid(&G[1], expand_kgrid(kgrid_2bit_512, 512, 8, 2), 512, 8, 43692, 2, 2);
    build_grid(&G[2], expand_kgrid(kgrid_2bit_1024, 1024, 8, 2), 1024, 8, 43692, 2, 1);
    build_grid(&G[3], expand_kgrid(kgrid_256, 256, 4, 3), 256, 4, 4096, 3, 2);
    build_grid(&G[4], expand_kgrid(kgrid_512, 512, 4, 3), 512, 4, 4096, 3, 3);
}
static const grid_data *grid(int which) {
    pthread_once(&grid_once, init_grids);
    return &G[which];
}

int oq_grid_info(int which, int32_t *grid_size, int32_t *kmap_size, int64_t *n_neighbours, int32_t *kmap_out,
                 uint16_t *neighbours_out) {
    if (which < 0 || which > 4) return OQ_EINVAL;
    const grid_data *g = grid(which);
    if (grid_size) *grid_size = g->grid_size;
    if (kmap_size) *kmap_size = g->kmap_size;
    if (n_neighbours) *n_neighbours = g->n_neighbours;
    if (kmap_out) memcpy(kmap_out, g->map, sizeof(int32_t) * (size_t)g->kmap_size);
    if (neighbours_out) memcpy(neighbours_out, g->neighbours, sizeof(uint16_t) * (size_t)g->n_neighbours);
    return OQ_OK;
}

/* quant_iq.rs:137-167; returns grid index or -1 if no finite candidate */
static int find_best_neighbour(const grid_data *g, int32_t map_val, const float *xval, const float *waux, float scale,
                               int8_t *ls) {
    int64_t off = (int64_t)(-map_val - 1);
    int n = g->neighbours[off];
    float best_d2 = 3.40282347e+38f;
    int best = -1;
    for (int t = 0; t < n; t++) {
        int j = g->neighbours[off + 1 + t];
        const int8_t *pg = g->grid[j];
        float d2 = 0.0f;
        for (int i = 0; i < g->dim; i++) {
            float diff = scale * (float)pg[i] - xval[i];
            d2 += waux[i] * diff * diff;
        }
        if (d2 < best_d2) { best_d2 = d2; best = j; }
    }
    if (best < 0) return -1;
    for (int i = 0; i < g->dim; i++) ls[i] = (int8_t)((g->grid[best][i] - 1) / 2);
    return best;
}

/* quant_iq.rs:170-241 */
static float make_qp_quants(int n, int nmax, const float *x, uint8_t *ls, const float *w) {
    float max = 0.0f;
    for (int i = 0; i < n; i++) max = rmaxf(max, x[i]);
    if (max < GROUP_MAX_EPS) {
        memset(ls, 0, (size_t)n);
        return 0.0f;
    }
    float iscale = (float)nmax / max;
    for (int i = 0; i < n; i++) ls[i] = (uint8_t)nearest_int(iscale * x[i]);
    float scale = 1.0f / iscale;
    float best_mse = 0.0f;
    for (int i = 0; i < n; i++) {
        float diff = x[i] - scale * (float)ls[i];
        best_mse += w[i] * diff * diff;
    }
    for (int is = -4; is <= 4; is++) {
        if (is == 0) continue;
        float iscale_is = (0.1f * (float)is + (float)nmax) / max;
        float scale_is = 1.0f / iscale_is;
        float mse = 0.0f;
        for (int i = 0; i < n; i++) {
            int32_t l = mini(nearest_int(iscale_is * x[i]), nmax);
            float diff = x[i] - scale_is * (float)l;
            mse += w[i] * diff * diff;
        }
        if (mse < best_mse) { best_mse = mse; iscale = iscale_is; }
    }
    float sumlx = 0.0f, suml2 = 0.0f;
    for (int i = 0; i < n; i++) {
        int32_t l = mini(nearest_int(iscale * x[i]), nmax);
        ls[i] = (uint8_t)l;
        sumlx += w[i] * x[i] * (float)l;
        suml2 += w[i] * (float)(l * l);
    }
    for (int it = 0; it < 5; it++) {
        int n_changed = 0;
        for (int i = 0; i < n; i++) {
            float wi = w[i];
            float li = (float)ls[i];
            float slx = sumlx - wi * x[i] * li;
            float sl2 = suml2 - wi * li * li;
            if (slx > 0.0f && sl2 > 0.0f) {
                int32_t new_l = mini(nearest_int(x[i] * sl2 / slx), nmax);
                if ((uint8_t)new_l != ls[i]) {
                    float slx2 = slx + wi * x[i] * (float)new_l;
                    float sl22 = sl2 + wi * (float)(new_l * new_l);
                    if (slx2 * slx2 * suml2 > sumlx * sumlx * sl22) {
                        ls[i] = (uint8_t)new_l;
                        sumlx = slx2;
                        suml2 = sl22;
                        n_changed++;
                    }
                }
            }
        }
        if (n_changed == 0) break;
    }
    return suml2 > 0.0f ? sumlx / suml2 : 0.0f;
}

/* quant_iq.rs:245-271 */
static uint8_t signs_with_parity(const float *xb, const float *weight, int k, float *xval) {
    int nflip = 0;
    uint8_t s = 0;
    for (int i = 0; i < 8; i++) {
        if (xb[8 * k + i] >= 0.0f) {
            xval[8 * k + i] = xb[8 * k + i];
        } else {
            xval[8 * k + i] = -xb[8 * k + i];
            nflip++;
            s |= (uint8_t)(1u << i);
        }
    }
    if (nflip % 2 != 0) {
        int imin = 0;
        float mn = weight[8 * k] * xb[8 * k] * xb[8 * k];
        for (int i = 1; i < 8; i++) {
            float ax = weight[8 * k + i] * xb[8 * k + i] * xb[8 * k + i];
            if (ax < mn) { mn = ax; imin = i; }
        }
        xval[8 * k + imin] = -xval[8 * k + imin];
        s ^= (uint8_t)(1u << imin);
    }
    return s & 127;
}

static inline float sum_sq(const float *x, int n) {
    float s = 0.0f;
    for (int i = 0; i < n; i++) s += x[i] * x[i];
    return s;
}
static inline float fold_max_from_first(const float *x, int n) {
    float m = x[0];
    for (int i = 0; i < n; i++) m = rmaxf(m, x[i]);
    return m;
}

/* ---------------- IQ2_XXS (quant_iq.rs:275-407) ---------------- */
static int enc_iq2_xxs(const float *x, int64_t n, const float *im, uint8_t *out) {
    const grid_data *g = grid(0);
    const int k_max_q = 3;
    static const float ones[32] = {1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1,
                                   1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1};
    for (int64_t ibl = 0; ibl < n / 256; ibl++) {
        const float *xbl = x + 256 * ibl;
        uint8_t *o = out + 66 * ibl;
        memset(o, 0, 66);
        float sigma2 = sum_sq(xbl, 256) / 256.0f;
        uint32_t q2[16] = {0};
        float max_scale = 0.0f;
        float scales[8];
        for (int ib = 0; ib < 8; ib++) {
            const float *xb = xbl + 32 * ib;
            const float *qw = im ? im + 256 * ibl + 32 * ib : ones;
            float weight[32], waux[32];
            for (int i = 0; i < 32; i++) {
                weight[i] = qw[i] * sqrtf(sigma2 + xb[i] * xb[i]);
                waux[i] = sqrtf(weight[i]);
            }
            float xval[32];
            uint8_t block_signs[4];
            for (int k = 0; k < 4; k++) block_signs[k] = signs_with_parity(xb, weight, k, xval);
            float max = fold_max_from_first(xval, 32);
            int8_t ls[32] = {0};
            if (max < GROUP_MAX_EPS) { scales[ib] = 0.0f; continue; }
            uint8_t lp[32];
            float scale = make_qp_quants(32, k_max_q + 1, xval, lp, weight);
            float eff_max = scale * (float)k_max_q;
            if (eff_max <= 0.0f) { scales[ib] = 0.0f; continue; }
            float best = 0.0f;
            int8_t laux[32];
            for (int is = -6; is <= 6; is++) {
                float id = (float)(2 * k_max_q - 1) + (float)is * 0.1f;
                id = id / eff_max;
                float this_scale = 1.0f / id;
                for (int k = 0; k < 4; k++) {
                    for (int i = 0; i < 8; i++)
                        laux[8 * k + i] = (int8_t)clampi(nearest_int(0.5f * (id * xval[8 * k + i] - 1.0f)), 0, k_max_q - 1);
                    int u = 0;
                    for (int i = 0; i < 8; i++) u |= laux[8 * k + i] << (2 * i);
                    if (g->map[u] < 0 &&
                        find_best_neighbour(g, g->map[u], xval + 8 * k, waux + 8 * k, this_scale, laux + 8 * k) < 0)
                        return OQ_ENONEIGHBOUR;
                }
                float sumqx = 0.0f, sumq2 = 0.0f;
                for (int i = 0; i < 32; i++) {
                    float q = (float)(2 * laux[i] + 1);
                    sumqx += weight[i] * xval[i] * q;
                    sumq2 += weight[i] * q * q;
                }
                if (sumq2 > 0.0f && sumqx * sumqx > best * sumq2) {
                    scale = sumqx / sumq2;
                    best = scale * sumqx;
                    memcpy(ls, laux, 32);
                }
            }
            if (scale > 0.0f) {
                float id = 1.0f / scale;
                for (int k = 0; k < 4; k++) {
                    int u = 0;
                    for (int i = 0; i < 8; i++) {
                        int32_t l = clampi(nearest_int(0.5f * (id * xval[8 * k + i] - 1.0f)), 0, k_max_q - 1);
                        u |= l << (2 * i);
                    }
                    int gi;
                    if (g->map[u] >= 0) {
                        gi = g->map[u];
                    } else {
                        gi = find_best_neighbour(g, g->map[u], xval + 8 * k, waux + 8 * k, scale, ls + 8 * k);
                        if (gi < 0) return OQ_ENONEIGHBOUR;
                    }
                    for (int i = 0; i < 8; i++) ls[8 * k + i] = (int8_t)((g->grid[gi][i] - 1) / 2);
                }
                float sumqx = 0.0f, sumq2 = 0.0f;
                for (int i = 0; i < 32; i++) {
                    float q = (float)(2 * ls[i] + 1);
                    sumqx += weight[i] * xval[i] * q;
                    sumq2 += weight[i] * q * q;
                }
                if (sumq2 > 0.0f) scale = sumqx / sumq2;
            }
            if (scale < 0.0f) {
                scale = -scale;
                for (int k = 0; k < 4; k++) block_signs[k] = (uint8_t)((~block_signs[k]) & 127);
            }
            for (int k = 0; k < 4; k++) {
                int u = 0;
                for (int i = 0; i < 8; i++) u |= ls[8 * k + i] << (2 * i);
                int32_t gi = g->map[u];
                if (gi < 0) return OQ_EOFFGRID;
                q2[2 * ib] |= (uint32_t)gi << (8 * k);
                q2[2 * ib + 1] |= (uint32_t)block_signs[k] << (7 * k);
            }
            scales[ib] = scale;
            max_scale = rmaxf(max_scale, scale);
        }
        if (max_scale == 0.0f) continue;
        float d = max_scale / 31.0f;
        put_f16(o, d);
        float id = 1.0f / d;
        for (int ib = 0; ib < 8; ib++) {
            int32_t l = clampi(nearest_int(0.5f * (id * scales[ib] - 1.0f)), 0, 15);
            q2[2 * ib + 1] |= (uint32_t)l << 28;
        }
        for (int i = 0; i < 16; i++) wr_u32(o + 2 + 4 * i, q2[i]);
    }
    return OQ_OK;
}

static void dec_iq2_xxs(const uint8_t *data, int64_t n, float *out) {
    for (int64_t b = 0; b < n / 256; b++) {
        const uint8_t *blk = data + 66 * b;
        float d = get_f16(blk);
        float *y = out + 256 * b;
        for (int ib32 = 0; ib32 < 8; ib32++) {
            uint32_t a0 = rd_u32(blk + 2 + 8 * ib32), a1 = rd_u32(blk + 6 + 8 * ib32);
            float db = d * (0.5f + (float)(a1 >> 28)) * 0.25f;
            for (int l = 0; l < 4; l++) {
                uint64_t gv = iq2xxs_grid[(a0 >> (8 * l)) & 255];
                uint8_t signs = ksigns_iq2xs[(a1 >> (7 * l)) & 127];
                for (int j = 0; j < 8; j++) {
                    float s = (signs & kmask_iq2xs[j]) ? -1.0f : 1.0f;
                    *y++ = db * (float)(uint8_t)(gv >> (8 * j)) * s;
                }
            }
        }
    }
}

/* ---------------- IQ2_XS (quant_iq.rs:430-563) ---------------- */
static int enc_iq2_xs(const float *x, int64_t n, const float *im, uint8_t *out) {
    const grid_data *g = grid(1);
    const int k_max_q = 3;
    static const float ones[16] = {1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1};
    for (int64_t ibl = 0; ibl < n / 256; ibl++) {
        const float *xbl = x + 256 * ibl;
        uint8_t *o = out + 74 * ibl;
        memset(o, 0, 74);
        float sigma2 = sum_sq(xbl, 256) / 256.0f;
        uint16_t q2[32] = {0};
        uint8_t sc[8] = {0};
        float max_scale = 0.0f;
        float scales[16];
        for (int ib = 0; ib < 16; ib++) {
            const float *xb = xbl + 16 * ib;
            const float *qw = im ? im + 256 * ibl + 16 * ib : ones;
            float weight[16], waux[16];
            for (int i = 0; i < 16; i++) {
                weight[i] = qw[i] * sqrtf(sigma2 + xb[i] * xb[i]);
                waux[i] = sqrtf(weight[i]);
            }
            float xval[16];
            uint8_t block_signs[2];
            for (int k = 0; k < 2; k++) block_signs[k] = signs_with_parity(xb, weight, k, xval);
            float max = fold_max_from_first(xval, 16);
            int8_t ls[16] = {0};
            if (max < GROUP_MAX_EPS) { scales[ib] = 0.0f; continue; }
            float best = 0.0f;
            float scale = max / (float)(2 * k_max_q - 1);
            int is_on_grid[2] = {1, 1};
            int8_t laux[16];
            for (int is = -9; is <= 9; is++) {
                float id = ((float)(2 * k_max_q - 1) + (float)is * 0.1f) / max;
                float this_scale = 1.0f / id;
                int aux[2] = {1, 1};
                for (int k = 0; k < 2; k++) {
                    for (int i = 0; i < 8; i++)
                        laux[8 * k + i] = (int8_t)clampi(nearest_int(0.5f * (id * xval[8 * k + i] - 1.0f)), 0, k_max_q - 1);
                    int u = 0;
                    for (int i = 0; i < 8; i++) u |= laux[8 * k + i] << (2 * i);
                    if (g->map[u] < 0) {
                        aux[k] = 0;
                        if (find_best_neighbour(g, g->map[u], xval + 8 * k, waux + 8 * k, this_scale, laux + 8 * k) < 0)
                            return OQ_ENONEIGHBOUR;
                    }
                }
                float sumqx = 0.0f, sumq2 = 0.0f;
                for (int i = 0; i < 16; i++) {
                    float q = (float)(2 * laux[i] + 1);
                    sumqx += weight[i] * xval[i] * q;
                    sumq2 += weight[i] * q * q;
                }
                if (sumq2 > 0.0f && sumqx * sumqx > best * sumq2) {
                    scale = sumqx / sumq2;
                    best = scale * sumqx;
                    memcpy(ls, laux, 16);
                    is_on_grid[0] = aux[0];
                    is_on_grid[1] = aux[1];
                }
            }
            int n_not = (!is_on_grid[0]) + (!is_on_grid[1]);
            if (n_not > 0 && scale > 0.0f) {
                float id = 1.0f / scale;
                for (int k = 0; k < 2; k++) {
                    if (is_on_grid[k]) continue;
                    int u = 0;
                    for (int i = 0; i < 8; i++) {
                        int32_t l = clampi(nearest_int(0.5f * (id * xval[8 * k + i] - 1.0f)), 0, k_max_q - 1);
                        u |= l << (2 * i);
                        ls[8 * k + i] = (int8_t)l;
                    }
                    if (g->map[u] < 0 &&
                        find_best_neighbour(g, g->map[u], xval + 8 * k, waux + 8 * k, scale, ls + 8 * k) < 0)
                        return OQ_ENONEIGHBOUR;
                }
                float sumqx = 0.0f, sumq2 = 0.0f;
                for (int i = 0; i < 16; i++) {
                    float q = (float)(2 * ls[i] + 1);
                    sumqx += weight[i] * xval[i] * q;
                    sumq2 += weight[i] * q * q;
                }
                if (sumq2 > 0.0f) scale = sumqx / sumq2;
            }
            if (scale < 0.0f) {
                scale = -scale;
                for (int k = 0; k < 2; k++) block_signs[k] = (uint8_t)((~block_signs[k]) & 127);
            }
            for (int k = 0; k < 2; k++) {
                int u = 0;
                for (int i = 0; i < 8; i++) u |= ls[8 * k + i] << (2 * i);
                int32_t gi = g->map[u];
                if (gi < 0) return OQ_EOFFGRID;
                q2[2 * ib + k] = (uint16_t)((uint32_t)gi | ((uint32_t)block_signs[k] << 9));
            }
            scales[ib] = scale;
            max_scale = rmaxf(max_scale, scale);
        }
        if (max_scale == 0.0f) continue;
        float d = max_scale / 31.0f;
        put_f16(o, d);
        float id = 1.0f / d;
        for (int ib = 0; ib < 16; ib++) {
            uint8_t l = (uint8_t)clampi(nearest_int(0.5f * (id * scales[ib] - 1.0f)), 0, 15);
            if (ib % 2 == 0) sc[ib / 2] = l;
            else sc[ib / 2] |= (uint8_t)(l << 4);
        }
        for (int i = 0; i < 32; i++) { o[2 + 2 * i] = (uint8_t)q2[i]; o[3 + 2 * i] = (uint8_t)(q2[i] >> 8); }
        memcpy(o + 66, sc, 8);
    }
    return OQ_OK;
}

static void dec_iq2_xs(const uint8_t *data, int64_t n, float *out) {
    for (int64_t b = 0; b < n / 256; b++) {
        const uint8_t *blk = data + 74 * b;
        float d = get_f16(blk);
        float *y = out + 256 * b;
        for (int ib32 = 0; ib32 < 8; ib32++) {
            uint8_t sc = blk[66 + ib32];
            float db[2] = {d * (0.5f + (float)(sc & 0xF)) * 0.25f, d * (0.5f + (float)(sc >> 4)) * 0.25f};
            for (int l = 0; l < 4; l++) {
                uint16_t q = (uint16_t)(blk[2 + 8 * ib32 + 2 * l] | (blk[3 + 8 * ib32 + 2 * l] << 8));
                uint64_t gv = iq2xs_grid[q & 511];
                uint8_t signs = ksigns_iq2xs[q >> 9];
                for (int j = 0; j < 8; j++) {
                    float s = (signs & kmask_iq2xs[j]) ? -1.0f : 1.0f;
                    *y++ = db[l / 2] * (float)(uint8_t)(gv >> (8 * j)) * s;
                }
            }
        }
    }
}

/* ---------------- IQ2_S (quant_iq.rs:589-730) ---------------- */
static int enc_iq2_s(const float *x, int64_t n, const float *im, uint8_t *out) {
    const grid_data *g = grid(2);
    const int k_max_q = 3;
    for (int64_t ibl = 0; ibl < n / 256; ibl++) {
        const float *xbl = x + 256 * ibl;
        uint8_t *o = out + 82 * ibl;
        memset(o, 0, 82);
        float sigma2 = 2.0f * sum_sq(xbl, 256) / 256.0f;
        float max_scale = 0.0f;
        float scales[16];
        for (int ib = 0; ib < 16; ib++) {
            const float *xb = xbl + 16 * ib;
            float weight[16], waux[16];
            for (int i = 0; i < 16; i++) {
                weight[i] = im ? im[256 * ibl + 16 * ib + i] * sqrtf(sigma2 + xb[i] * xb[i])
                               : 0.25f * sigma2 + xb[i] * xb[i];
                waux[i] = sqrtf(weight[i]);
            }
            float xval[16];
            uint8_t block_signs[2];
            for (int k = 0; k < 2; k++) {
                uint8_t s = 0;
                for (int i = 0; i < 8; i++) {
                    if (xb[8 * k + i] >= 0.0f) xval[8 * k + i] = xb[8 * k + i];
                    else { xval[8 * k + i] = -xb[8 * k + i]; s |= (uint8_t)(1u << i); }
                }
                block_signs[k] = s;
            }
            float max = fold_max_from_first(xval, 16);
            int8_t ls[16] = {0};
            if (max < GROUP_MAX_EPS_IQ2_S) { scales[ib] = 0.0f; continue; }
            float best = 0.0f;
            float scale = max / (float)(2 * k_max_q - 1);
            int is_on_grid[2] = {1, 1};
            int8_t laux[16];
            for (int is = -9; is <= 9; is++) {
                float id = ((float)(2 * k_max_q - 1) + (float)is * 0.1f) / max;
                float this_scale = 1.0f / id;
                int aux[2] = {1, 1};
                for (int k = 0; k < 2; k++) {
                    for (int i = 0; i < 8; i++)
                        laux[8 * k + i] = (int8_t)clampi(nearest_int(0.5f * (id * xval[8 * k + i] - 1.0f)), 0, k_max_q - 1);
                    int u = 0;
                    for (int i = 0; i < 8; i++) u |= laux[8 * k + i] << (2 * i);
                    if (g->map[u] < 0) {
                        aux[k] = 0;
                        if (find_best_neighbour(g, g->map[u], xval + 8 * k, waux + 8 * k, this_scale, laux + 8 * k) < 0)
                            return OQ_ENONEIGHBOUR;
                    }
                }
                float sumqx = 0.0f, sumq2 = 0.0f;
                for (int i = 0; i < 16; i++) {
                    float q = (float)(2 * laux[i] + 1);
                    sumqx += weight[i] * xval[i] * q;
                    sumq2 += weight[i] * q * q;
                }
                if (sumq2 > 0.0f && sumqx * sumqx > best * sumq2) {
                    scale = sumqx / sumq2;
                    best = scale * sumqx;
                    memcpy(ls, laux, 16);
                    is_on_grid[0] = aux[0];
                    is_on_grid[1] = aux[1];
                }
            }
            int n_not = (!is_on_grid[0]) + (!is_on_grid[1]);
            if (n_not > 0 && scale > 0.0f) {
                float id = 1.0f / scale;
                for (int k = 0; k < 2; k++) {
                    if (is_on_grid[k]) continue;
                    int u = 0;
                    for (int i = 0; i < 8; i++) {
                        int32_t l = clampi(nearest_int(0.5f * (id * xval[8 * k + i] - 1.0f)), 0, k_max_q - 1);
                        u |= l << (2 * i);
                        ls[8 * k + i] = (int8_t)l;
                    }
                    if (g->map[u] < 0 &&
                        find_best_neighbour(g, g->map[u], xval + 8 * k, waux + 8 * k, scale, ls + 8 * k) < 0)
                        return OQ_ENONEIGHBOUR;
                }
                float sumqx = 0.0f, sumq2 = 0.0f;
                for (int i = 0; i < 16; i++) {
                    float q = (float)(2 * ls[i] + 1);
                    sumqx += weight[i] * xval[i] * q;
                    sumq2 += weight[i] * q * q;
                }
                if (sumq2 > 0.0f) scale = sumqx / sumq2;
            }
            if (scale < 0.0f) {
                scale = -scale;
                for (int k = 0; k < 2; k++) block_signs[k] = (uint8_t)~block_signs[k];
            }
            for (int k = 0; k < 2; k++) {
                int u = 0;
                for (int i = 0; i < 8; i++) u |= ls[8 * k + i] << (2 * i);
                int32_t gi = g->map[u];
                if (gi < 0) return OQ_EOFFGRID;
                int i8v = 2 * ib + k;
                o[2 + i8v] = (uint8_t)(gi & 255);
                o[2 + 64 + i8v / 4] |= (uint8_t)((gi >> 8) << (2 * (i8v % 4)));
                o[2 + 32 + i8v] = block_signs[k];
            }
            scales[ib] = scale;
            max_scale = rmaxf(max_scale, scale);
        }
        if (max_scale == 0.0f) continue;
        float d = max_scale / 31.0f;
        put_f16(o, d * 0.9875f);
        float id = 1.0f / d;
        for (int ib = 0; ib < 16; ib++) {
            uint8_t l = (uint8_t)clampi(nearest_int(0.5f * (id * scales[ib] - 1.0f)), 0, 15);
            int so = 2 + 64 + 8 + ib / 2;
            if (ib % 2 == 0) o[so] = l;
            else o[so] |= (uint8_t)(l << 4);
        }
    }
    return OQ_OK;
}

static void dec_iq2_s(const uint8_t *data, int64_t n, float *out) {
    for (int64_t b = 0; b < n / 256; b++) {
        const uint8_t *blk = data + 82 * b;
        float d = get_f16(blk);
        const uint8_t *qs = blk + 2, *qh = blk + 66, *sc = blk + 74;
        float *y = out + 256 * b;
        for (int ib32 = 0; ib32 < 8; ib32++) {
            float db[2] = {d * (0.5f + (float)(sc[ib32] & 0xF)) * 0.25f, d * (0.5f + (float)(sc[ib32] >> 4)) * 0.25f};
            for (int l = 0; l < 4; l++) {
                int idx = qs[4 * ib32 + l] | ((qh[ib32] << (8 - 2 * l)) & 0x300);
                uint64_t gv = iq2s_grid[idx];
                uint8_t signs = qs[32 + 4 * ib32 + l];
                for (int j = 0; j < 8; j++) {
                    float s = (signs & kmask_iq2xs[j]) ? -1.0f : 1.0f;
                    *y++ = db[l / 2] * (float)(uint8_t)(gv >> (8 * j)) * s;
                }
            }
        }
    }
}

/* ---------------- IQ3_XXS / IQ3_S (quant_iq.rs:758-935) ---------------- */
static int enc_iq3(int five, const float *x, int64_t n, const float *im, uint8_t *out) {
    const grid_data *g = grid(five ? 4 : 3);
    const int k_max_q = 8;
    int64_t block_bytes = five ? 110 : 98;
    int is_lo = five ? -9 : -15, is_hi = five ? 9 : 15;
    float is_step = 0.2f;
    for (int64_t ibl = 0; ibl < n / 256; ibl++) {
        const float *xbl = x + 256 * ibl;
        uint8_t *o = out + block_bytes * ibl;
        memset(o, 0, (size_t)block_bytes);
        float sigma2 = 2.0f * sum_sq(xbl, 256) / 256.0f;
        float max_scale = 0.0f;
        float scales[8];
        uint32_t sas[8] = {0};
        for (int ib = 0; ib < 8; ib++) {
            const float *xb = xbl + 32 * ib;
            float weight[32], waux[32];
            for (int i = 0; i < 32; i++) {
                weight[i] = im ? im[256 * ibl + 32 * ib + i] * sqrtf(sigma2 + xb[i] * xb[i]) : xb[i] * xb[i];
                waux[i] = sqrtf(weight[i]);
            }
            float xval[32];
            uint8_t block_signs[4];
            for (int k = 0; k < 4; k++) {
                if (five) {
                    uint8_t s = 0;
                    for (int i = 0; i < 8; i++) {
                        if (xb[8 * k + i] >= 0.0f) xval[8 * k + i] = xb[8 * k + i];
                        else { xval[8 * k + i] = -xb[8 * k + i]; s |= (uint8_t)(1u << i); }
                    }
                    block_signs[k] = s;
                } else {
                    block_signs[k] = signs_with_parity(xb, weight, k, xval);
                }
            }
            float max = fold_max_from_first(xval, 32);
            int8_t ls[32] = {0};
            float eps = five ? 0.0f : GROUP_MAX_EPS_IQ3_XXS;
            if (max <= eps) { scales[ib] = 0.0f; continue; }
            float best = 0.0f;
            float scale = max / (float)(2 * k_max_q - 1);
            int is_on_grid[8];
            for (int k = 0; k < 8; k++) is_on_grid[k] = !five;
            int8_t laux[32];
            for (int is = is_lo; is <= is_hi; is++) {
                float id = ((float)(2 * k_max_q - 1) + (float)is * is_step) / max;
                float this_scale = 1.0f / id;
                int aux[8];
                for (int k = 0; k < 8; k++) {
                    aux[k] = 1;
                    for (int i = 0; i < 4; i++)
                        laux[4 * k + i] = (int8_t)clampi(nearest_int(0.5f * (id * xval[4 * k + i] - 1.0f)), 0, k_max_q - 1);
                    int u = 0;
                    for (int i = 0; i < 4; i++) u |= laux[4 * k + i] << (3 * i);
                    if (g->map[u] < 0) {
                        aux[k] = 0;
                        if (find_best_neighbour(g, g->map[u], xval + 4 * k, waux + 4 * k, this_scale, laux + 4 * k) < 0)
                            return OQ_ENONEIGHBOUR;
                    }
                }
                float sumqx = 0.0f, sumq2 = 0.0f;
                for (int i = 0; i < 32; i++) {
                    float q = (float)(2 * laux[i] + 1);
                    sumqx += weight[i] * xval[i] * q;
                    sumq2 += weight[i] * q * q;
                }
                if (sumq2 > 0.0f && sumqx * sumqx > best * sumq2) {
                    scale = sumqx / sumq2;
                    best = scale * sumqx;
                    memcpy(ls, laux, 32);
                    for (int k = 0; k < 8; k++) is_on_grid[k] = aux[k];
                }
            }
            int n_not = 0;
            for (int k = 0; k < 8; k++) n_not += !is_on_grid[k];
            if (n_not > 0 && scale > 0.0f) {
                float id = 1.0f / scale;
                for (int k = 0; k < 8; k++) {
                    if (!five && is_on_grid[k]) continue;
                    int u = 0;
                    for (int i = 0; i < 4; i++) {
                        int32_t l = clampi(nearest_int(0.5f * (id * xval[4 * k + i] - 1.0f)), 0, k_max_q - 1);
                        u |= l << (3 * i);
                    }
                    int gi;
                    if (g->map[u] >= 0) {
                        gi = g->map[u];
                    } else {
                        gi = find_best_neighbour(g, g->map[u], xval + 4 * k, waux + 4 * k, scale, ls + 4 * k);
                        if (gi < 0) return OQ_ENONEIGHBOUR;
                    }
                    for (int i = 0; i < 4; i++) ls[4 * k + i] = (int8_t)((g->grid[gi][i] - 1) / 2);
                }
                float sumqx = 0.0f, sumq2 = 0.0f;
                for (int i = 0; i < 32; i++) {
                    float q = (float)(2 * ls[i] + 1);
                    sumqx += weight[i] * xval[i] * q;
                    sumq2 += weight[i] * q * q;
                }
                if (sumq2 > 0.0f) scale = sumqx / sumq2;
            }
            if (scale < 0.0f) {
                scale = -scale;
                for (int k = 0; k < 4; k++) block_signs[k] = five ? (uint8_t)~block_signs[k] : (uint8_t)((~block_signs[k]) & 127);
            }
            for (int k = 0; k < 8; k++) {
                int u = 0;
                for (int i = 0; i < 4; i++) u |= ls[4 * k + i] << (3 * i);
                int32_t gi = g->map[u];
                if (gi < 0) return OQ_EOFFGRID;
                if (five) {
                    o[2 + 8 * ib + k] = (uint8_t)(gi & 255);
                    o[2 + 64 + ib] |= (uint8_t)((gi >> 8) << k);
                } else {
                    o[2 + 8 * ib + k] = (uint8_t)gi;
                }
            }
            if (five) {
                for (int k = 0; k < 4; k++) o[2 + 64 + 8 + 4 * ib + k] = block_signs[k];
            } else {
                sas[ib] = (uint32_t)block_signs[0] | ((uint32_t)block_signs[1] << 7) | ((uint32_t)block_signs[2] << 14) |
                          ((uint32_t)block_signs[3] << 21);
            }
            scales[ib] = scale;
            max_scale = rmaxf(max_scale, scale);
        }
        if (max_scale == 0.0f) continue;
        float d = max_scale / 31.0f;
        float fudge = five ? 1.033f : 1.0125f;
        put_f16(o, d * fudge);
        float id = 1.0f / d;
        if (five) {
            for (int ib = 0; ib < 8; ib += 2) {
                uint8_t l1 = (uint8_t)clampi(nearest_int(0.5f * (id * scales[ib] - 1.0f)), 0, 15);
                uint8_t l2 = (uint8_t)clampi(nearest_int(0.5f * (id * scales[ib + 1] - 1.0f)), 0, 15);
                o[2 + 64 + 8 + 32 + ib / 2] = (uint8_t)(l1 | (l2 << 4));
            }
        } else {
            for (int ib = 0; ib < 8; ib++) {
                int32_t l = clampi(nearest_int(0.5f * (id * scales[ib] - 1.0f)), 0, 15);
                sas[ib] |= (uint32_t)l << 28;
            }
            for (int i = 0; i < 8; i++) wr_u32(o + 2 + 64 + 4 * i, sas[i]);
        }
    }
    return OQ_OK;
}

static void dec_iq3_xxs(const uint8_t *data, int64_t n, float *out) {
    for (int64_t b = 0; b < n / 256; b++) {
        const uint8_t *blk = data + 98 * b;
        float d = get_f16(blk);
        const uint8_t *qs = blk + 2;
        float *y = out + 256 * b;
        for (int ib32 = 0; ib32 < 8; ib32++) {
            uint32_t aux = rd_u32(blk + 66 + 4 * ib32);
            float db = d * (0.5f + (float)(aux >> 28)) * 0.5f;
            for (int l = 0; l < 4; l++) {
                uint8_t signs = ksigns_iq2xs[(aux >> (7 * l)) & 127];
                uint32_t g1 = iq3xxs_grid[qs[8 * ib32 + 2 * l]], g2 = iq3xxs_grid[qs[8 * ib32 + 2 * l + 1]];
                for (int j = 0; j < 4; j++) {
                    float s = (signs & kmask_iq2xs[j]) ? -1.0f : 1.0f;
                    *y++ = db * (float)(uint8_t)(g1 >> (8 * j)) * s;
                }
                for (int j = 0; j < 4; j++) {
                    float s = (signs & kmask_iq2xs[j + 4]) ? -1.0f : 1.0f;
                    *y++ = db * (float)(uint8_t)(g2 >> (8 * j)) * s;
                }
            }
        }
    }
}

static void dec_iq3_s(const uint8_t *data, int64_t n, float *out) {
    for (int64_t b = 0; b < n / 256; b++) {
        const uint8_t *blk = data + 110 * b;
        float d = get_f16(blk);
        const uint8_t *qs = blk + 2, *qh = blk + 66, *signs = blk + 74, *sc = blk + 106;
        float *y = out + 256 * b;
        for (int ib32 = 0; ib32 < 8; ib32++) {
            float db = ib32 % 2 == 0 ? d * (float)(1 + 2 * (sc[ib32 / 2] & 0xF)) : d * (float)(1 + 2 * (sc[ib32 / 2] >> 4));
            for (int l = 0; l < 4; l++) {
                int i1 = qs[8 * ib32 + 2 * l] | ((qh[ib32] << (8 - 2 * l)) & 256);
                int i2 = qs[8 * ib32 + 2 * l + 1] | ((qh[ib32] << (7 - 2 * l)) & 256);
                uint32_t g1 = iq3s_grid[i1], g2 = iq3s_grid[i2];
                uint8_t sg = signs[4 * ib32 + l];
                for (int j = 0; j < 4; j++) {
                    float s = (sg & kmask_iq2xs[j]) ? -1.0f : 1.0f;
                    *y++ = db * (float)(uint8_t)(g1 >> (8 * j)) * s;
                }
                for (int j = 0; j < 4; j++) {
                    float s = (sg & kmask_iq2xs[j + 4]) ? -1.0f : 1.0f;
                    *y++ = db * (float)(uint8_t)(g2 >> (8 * j)) * s;
                }
            }
        }
    }
}

/* ---------------- IQ4_NL / IQ4_XS (quant_iq.rs:1002-1189) ---------------- */
static int best_index_int8(const int8_t *vals, float x) {
    if (x <= (float)vals[0]) return 0;
    if (x >= (float)vals[15]) return 15;
    int ml = 0, mu = 15;
    while (mu - ml > 1) {
        int mav = (ml + mu) / 2;
        if (x < (float)vals[mav]) mu = mav;
        else ml = mav;
    }
    return x - (float)vals[mu - 1] < (float)vals[mu] - x ? mu - 1 : mu;
}

static void iq4_impl(int super_block, const float *x, const float *qw, uint8_t *d_out, uint8_t *q4, uint8_t *sh,
                     uint8_t *sl) {
    const int8_t *values = kvalues_iq4nl;
    const int ntry = 7;
    float sigma2 = 2.0f * sum_sq(x, super_block) / (float)super_block;
    int nb = super_block / 32;
    uint8_t ls_all[256] = {0};
    float scales[8];
    float max_scale = 0.0f, amax_scale = 0.0f;
    for (int ib = 0; ib < nb; ib++) {
        const float *xb = x + 32 * ib;
        float weight[32];
        for (int j = 0; j < 32; j++) weight[j] = qw ? qw[32 * ib + j] * sqrtf(sigma2 + xb[j] * xb[j]) : xb[j] * xb[j];
        float amax = 0.0f, max = 0.0f;
        for (int j = 0; j < 32; j++)
            if (fabsf(xb[j]) > amax) { amax = fabsf(xb[j]); max = xb[j]; }
        if (amax < GROUP_MAX_EPS) { scales[ib] = 0.0f; continue; }
        float d = -max / (float)values[0];
        float id = 1.0f / d;
        float sumqx = 0.0f, sumq2 = 0.0f;
        for (int j = 0; j < 32; j++) {
            int l = best_index_int8(values, id * xb[j]);
            ls_all[32 * ib + j] = (uint8_t)l;
            float q = (float)values[l];
            sumqx += weight[j] * q * xb[j];
            sumq2 += weight[j] * q * q;
        }
        d = sumq2 > 0.0f ? sumqx / sumq2 : 0.0f;
        float best = d * sumqx;
        for (int itry = -ntry; itry <= ntry; itry++) {
            id = ((float)itry + (float)values[0]) / max;
            sumqx = 0.0f;
            sumq2 = 0.0f;
            for (int j = 0; j < 32; j++) {
                int l = best_index_int8(values, id * xb[j]);
                float q = (float)values[l];
                sumqx += weight[j] * q * xb[j];
                sumq2 += weight[j] * q * q;
            }
            if (sumq2 > 0.0f && sumqx * sumqx > best * sumq2) {
                d = sumqx / sumq2;
                best = d * sumqx;
            }
        }
        scales[ib] = d;
        if (fabsf(d) > amax_scale) { amax_scale = fabsf(d); max_scale = d; }
    }
    if (nb > 1) {
        float d = -max_scale / 32.0f;
        put_f16(d_out, d);
        float id = d != 0.0f ? 1.0f / d : 0.0f;
        uint16_t h16 = 0;
        for (int ib = 0; ib < nb; ib++) {
            int32_t l = clampi(nearest_int(id * scales[ib]), -32, 31);
            float dl = d * (float)l;
            float idl = dl != 0.0f ? 1.0f / dl : 0.0f;
            const float *xb = x + 32 * ib;
            for (int j = 0; j < 32; j++) ls_all[32 * ib + j] = (uint8_t)best_index_int8(values, idl * xb[j]);
            uint8_t lu = (uint8_t)(l + 32);
            if (ib % 2 == 0) sl[ib / 2] = lu & 0xF;
            else sl[ib / 2] |= (uint8_t)((lu & 0xF) << 4);
            h16 |= (uint16_t)((lu >> 4) << (2 * ib));
        }
        sh[0] = (uint8_t)h16;
        sh[1] = (uint8_t)(h16 >> 8);
    } else {
        put_f16(d_out, scales[0]);
        float id = scales[0] != 0.0f ? 1.0f / scales[0] : 0.0f;
        for (int j = 0; j < super_block; j++) ls_all[j] = (uint8_t)best_index_int8(values, id * x[j]);
    }
    for (int i = 0; i < super_block / 32; i++)
        for (int j = 0; j < 16; j++) q4[16 * i + j] = (uint8_t)(ls_all[32 * i + j] | (ls_all[32 * i + 16 + j] << 4));
}

static void enc_iq4_nl(const float *x, int64_t n, const float *im, uint8_t *out) {
    for (int64_t ib = 0; ib < n / 32; ib++) {
        uint8_t *o = out + 18 * ib;
        memset(o, 0, 18);
        iq4_impl(32, x + 32 * ib, im ? im + 32 * ib : NULL, o, o + 2, NULL, NULL);
    }
}
static void enc_iq4_xs(const float *x, int64_t n, const float *im, uint8_t *out) {
    for (int64_t ibl = 0; ibl < n / 256; ibl++) {
        uint8_t *o = out + 136 * ibl;
        memset(o, 0, 136);
        iq4_impl(256, x + 256 * ibl, im ? im + 256 * ibl : NULL, o, o + 8, o + 2, o + 4);
    }
}
static void dec_iq4_nl(const uint8_t *data, int64_t n, float *out) {
    for (int64_t b = 0; b < n / 32; b++) {
        const uint8_t *blk = data + 18 * b;
        float d = get_f16(blk);
        const uint8_t *qs = blk + 2;
        for (int j = 0; j < 16; j++) out[32 * b + j] = d * (float)kvalues_iq4nl[qs[j] & 0xF];
        for (int j = 0; j < 16; j++) out[32 * b + 16 + j] = d * (float)kvalues_iq4nl[qs[j] >> 4];
    }
}
static void dec_iq4_xs(const uint8_t *data, int64_t n, float *out) {
    for (int64_t b = 0; b < n / 256; b++) {
        const uint8_t *blk = data + 136 * b;
        float d = get_f16(blk);
        uint16_t sh = (uint16_t)(blk[2] | (blk[3] << 8));
        const uint8_t *sl = blk + 4, *qs = blk + 8;
        float *y = out + 256 * b;
        for (int ib = 0; ib < 8; ib++) {
            int ls = ((sl[ib / 2] >> (4 * (ib % 2))) & 0xF) | (((sh >> (2 * ib)) & 3) << 4);
            float dl = d * (float)(ls - 32);
            for (int j = 0; j < 16; j++) y[32 * ib + j] = dl * (float)kvalues_iq4nl[qs[16 * ib + j] & 0xF];
            for (int j = 0; j < 16; j++) y[32 * ib + 16 + j] = dl * (float)kvalues_iq4nl[qs[16 * ib + j] >> 4];
        }
    }
}

/* ---------------- public API (quant.rs:543-630) ---------------- */

int oq_encode_row(uint32_t type, const float *x, int64_t n, const float *im, uint8_t *out) {
    if (oq_row_bytes(type, n) < 0) return OQ_EINVAL;
    float sigma2 = row_sigma2(x, n);
    switch (type) {
    case T_F32: memcpy(out, x, sizeof(float) * (size_t)n); return OQ_OK;
    case T_F16: for (int64_t i = 0; i < n; i++) put_f16(out + 2 * i, x[i]); return OQ_OK;
    case T_BF16:
        for (int64_t i = 0; i < n; i++) {
            uint32_t b;
            memcpy(&b, &x[i], 4);
            out[2 * i] = (uint8_t)(b >> 16);
            out[2 * i + 1] = (uint8_t)(b >> 24);
        }
        return OQ_OK;
    case T_Q8_0: enc_q8_0(x, n, out); return OQ_OK;
    case T_Q4_0: enc_q4_0(x, n, im, sigma2, out); return OQ_OK;
    case T_Q4_1: enc_q4_1(x, n, im, sigma2, out); return OQ_OK;
    case T_Q5_0: enc_q5_0(x, n, im, sigma2, out); return OQ_OK;
    case T_Q5_1: enc_q5_1(x, n, im, sigma2, out); return OQ_OK;
    case T_Q6_K: enc_q6_k(x, n, im, sigma2, out); return OQ_OK;
    case T_Q2_K: enc_q2_k(x, n, im, sigma2, out); return OQ_OK;
    case T_Q3_K: enc_q3_k(x, n, im, sigma2, out); return OQ_OK;
    case T_Q4_K: enc_qk45(x, n, im, sigma2, 15, out); return OQ_OK;
    case T_Q5_K: enc_qk45(x, n, im, sigma2, 31, out); return OQ_OK;
    case T_IQ2_XXS: return enc_iq2_xxs(x, n, im, out);
    case T_IQ2_XS: return enc_iq2_xs(x, n, im, out);
    case T_IQ2_S: return enc_iq2_s(x, n, im, out);
    case T_IQ3_XXS: return enc_iq3(0, x, n, im, out);
    case T_IQ3_S: return enc_iq3(1, x, n, im, out);
    case T_IQ4_NL: enc_iq4_nl(x, n, im, out); return OQ_OK;
    case T_IQ4_XS: enc_iq4_xs(x, n, im, out); return OQ_OK;
    default: return OQ_EINVAL;
    }
}

int oq_decode_row(uint32_t type, const uint8_t *data, int64_t n, float *out) {
    if (oq_row_bytes(type, n) < 0) return OQ_EINVAL;
    switch (type) {
    case T_F32: memcpy(out, data, sizeof(float) * (size_t)n); return OQ_OK;
    case T_F16: for (int64_t i = 0; i < n; i++) out[i] = get_f16(data + 2 * i); return OQ_OK;
    case T_BF16:
        for (int64_t i = 0; i < n; i++) {
            uint32_t b = ((uint32_t)data[2 * i] | ((uint32_t)data[2 * i + 1] << 8)) << 16;
            memcpy(&out[i], &b, 4);
        }
        return OQ_OK;
    case T_Q8_0: dec_q8_0(data, n, out); return OQ_OK;
    case T_Q4_0: dec_q4_0(data, n, out); return OQ_OK;
    case T_Q4_1: dec_q4_1(data, n, out); return OQ_OK;
    case T_Q5_0: dec_q5_0(data, n, out); return OQ_OK;
    case T_Q5_1: dec_q5_1(data, n, out); return OQ_OK;
    case T_Q6_K: dec_q6_k(data, n, out); return OQ_OK;
    case T_Q2_K: dec_q2_k(data, n, out); return OQ_OK;
    case T_Q3_K: dec_q3_k(data, n, out); return OQ_OK;
    case T_Q4_K: dec_q4_k(data, n, out); return OQ_OK;
    case T_Q5_K: dec_q5_k(data, n, out); return OQ_OK;
    case T_IQ2_XXS: dec_iq2_xxs(data, n, out); return OQ_OK;
    case T_IQ2_XS: dec_iq2_xs(data, n, out); return OQ_OK;
    case T_IQ2_S: dec_iq2_s(data, n, out); return OQ_OK;
    case T_IQ3_XXS: dec_iq3_xxs(data, n, out); return OQ_OK;
    case T_IQ3_S: dec_iq3_s(data, n, out); return OQ_OK;
    case T_IQ4_NL: dec_iq4_nl(data, n, out); return OQ_OK;
    case T_IQ4_XS: dec_iq4_xs(data, n, out); return OQ_OK;
    default: return OQ_EINVAL;
    }
}

int oq_row_error(uint32_t type, const float *x, int64_t n, const float *im, double *err) {
    int64_t rb = oq_row_bytes(type, n);
    if (rb < 0) return OQ_EINVAL;
    uint8_t *enc = malloc((size_t)rb + 1);
    float *dec = malloc(sizeof(float) * (size_t)n + 1);
    int rc = oq_encode_row(type, x, n, im, enc);
    if (rc == OQ_OK) rc = oq_decode_row(type, enc, n, dec);
    if (rc == OQ_OK) {
        double e = 0.0;
        for (int64_t i = 0; i < n; i++) {
            double w = im ? (double)im[i] : 1.0;
            double d = (double)(x[i] - dec[i]);
            e += w * d * d;
        }
        *err = e;
    }
    free(enc);
    free(dec);
    return rc;
}

#ifndef SH_OPCOUNT
/* ---------------- tensor drivers (main.rs:663-686, 549-563) ---------------- */

/* imatrix.rs:124-141 row_slice */
static const float *row_slice(const float *im, int64_t im_len, int64_t ne0, int64_t rows_per_mat, int64_t row) {
    if (!im) return NULL;
    if (im_len == ne0) return im;
    if (rows_per_mat > 0 && ne0 > 0 && im_len % ne0 == 0) {
        int64_t mat = row / rows_per_mat;
        int64_t n_mats = im_len / ne0;
        int64_t m = mat < n_mats - 1 ? mat : n_mats - 1;
        return im + m * ne0;
    }
    return NULL;
}

typedef struct {
    uint32_t type;
    const uint16_t *src;
    int64_t n_rows, ne0;
    const float *im;
    int64_t im_len, rows_per_mat, row_step, n_items, chunk;
    uint8_t *dst;
    double *err;
    atomic_long next;
    atomic_int rc;
} job_t;

static void *worker(void *arg) {
    job_t *j = (job_t *)arg;
    int64_t rb = oq_row_bytes(j->type, j->ne0);
    float *row = malloc(sizeof(float) * (size_t)j->ne0 + 4);
    for (;;) {
        int64_t c0 = atomic_fetch_add(&j->next, j->chunk);
        if (c0 >= j->n_items) break;
        int64_t c1 = c0 + j->chunk < j->n_items ? c0 + j->chunk : j->n_items;
        for (int64_t it = c0; it < c1; it++) {
            int64_t r = j->dst ? it : it * j->row_step;
            const uint16_t *s = j->src + r * j->ne0;
            for (int64_t i = 0; i < j->ne0; i++) {
                uint32_t b = (uint32_t)s[i] << 16;
                memcpy(&row[i], &b, 4);
            }
            const float *ims = row_slice(j->im, j->im_len, j->ne0, j->rows_per_mat, r);
            int rc = j->dst ? oq_encode_row(j->type, row, j->ne0, ims, j->dst + r * rb)
                            : oq_row_error(j->type, row, j->ne0, ims, &j->err[it]);
            if (rc != OQ_OK) atomic_store(&j->rc, rc);
        }
    }
    free(row);
    return NULL;
}

static int run_job(job_t *j, int n_threads) {
    if (n_threads < 1) n_threads = 1;
    atomic_init(&j->next, 0);
    atomic_init(&j->rc, OQ_OK);
    /* main.rs:671: chunk = clamp(n_rows / (threads * 4), 1, 512) */
    int64_t chunk = j->n_items / ((int64_t)n_threads * 4);
    j->chunk = chunk < 1 ? 1 : (chunk > 512 ? 512 : chunk);
    if (n_threads == 1) {
        worker(j);
        return atomic_load(&j->rc);
    }
    pthread_t *th = malloc(sizeof(pthread_t) * (size_t)n_threads);
    for (int t = 0; t < n_threads; t++) pthread_create(&th[t], NULL, worker, j);
    for (int t = 0; t < n_threads; t++) pthread_join(th[t], NULL);
    free(th);
    return atomic_load(&j->rc);
}

int oq_encode_tensor_bf16(uint32_t type, const uint16_t *src, int64_t n_rows, int64_t ne0, const float *im,
                          int64_t im_len, int64_t rows_per_mat, uint8_t *dst, int n_threads) {
    if (oq_row_bytes(type, ne0) < 0 || n_rows < 0) return OQ_EINVAL;
    job_t j = {.type = type, .src = src, .n_rows = n_rows, .ne0 = ne0, .im = im, .im_len = im_len,
               .rows_per_mat = rows_per_mat, .row_step = 1, .n_items = n_rows, .dst = dst, .err = NULL};
    return run_job(&j, n_threads);
}

int oq_row_errors_bf16(uint32_t type, const uint16_t *src, int64_t n_rows, int64_t ne0, const float *im,
                       int64_t im_len, int64_t rows_per_mat, int64_t row_step, double *err, int n_threads) {
    if (oq_row_bytes(type, ne0) < 0 || n_rows < 0 || row_step < 1) return OQ_EINVAL;
    int64_t n_items = (n_rows + row_step - 1) / row_step;
    job_t j = {.type = type, .src = src, .n_rows = n_rows, .ne0 = ne0, .im = im, .im_len = im_len,
               .rows_per_mat = rows_per_mat, .row_step = row_step, .n_items = n_items, .dst = NULL, .err = err};
    return run_job(&j, n_threads);
}
#endif /* SH_OPCOUNT */
