// IQ codebook encoders (src/quant_iq.rs) for sm_100a.
//
// One warp per 256-element super-block.  The per-block scale trials of the
// reference are independent given the block's weights, so every
// (block, trial) pair is a lane job.  A job rounds its groups to the lattice;
// the groups that land off the grid become search tasks, and each task's
// neighbour list is scanned by a group of lanes together (the lists' lengths
// vary, so one lane per list would serialise the warp on the longest).  The
// reference's sequential `sumqx^2 > best*sumq2` chain over the trials is then
// replayed by one lane per block.  Lattice lookups use the compact kmap
// staged in shared memory; neighbour lists are read through the read-only
// cache.
#include <algorithm>
#include <cfloat>

#include "iq_tables.h"
#include "fuse.cuh"
#include "kernels.cuh"

namespace shc {

// ---------------------------------------------------------------------------
// IQ4_NL / IQ4_XS (quant_iq.rs:1002-1157)
// ---------------------------------------------------------------------------
__device__ const float d_kv_f[16] = {-127.f, -104.f, -83.f, -65.f, -49.f, -35.f, -22.f, -10.f,
                                     1.f,    13.f,   25.f,  38.f,  53.f,  69.f,  89.f,  113.f};

// best_index_int8 (quant_iq.rs:1002-1024).  For x strictly inside
// (v0, v15) the binary search ends at the unique mu with v[mu-1] <= x < v[mu];
// the codebook values are integers, so v[k] <= x <=> v[k] <= floor(x) and
// mu = 1 + cnt[floor(x)], with cnt[f] = #{k in 1..14 : v[k] <= f}.
// Outside, the end pairs keep the answer: for x <= -127 the pair (v0, v1)
// picks v0, for x >= 113 the pair (v14, v15) picks v15.  The table covers
// floor(x) in [-136, 135]; floor() is read from the mantissa of
// RD(x + 1.5*2^23) (no conversion instruction), slot = floor(x) + 136.
//
// Two entry forms:
//  - clamped (any x): fminf before fmaxf clamps to [-128, 127] and sends NaN
//    to 127, hence v15, where the reference's search ends for NaN;
//  - bounded (x in [-136, 136) or NaN, as the trial products id*x are: |id|
//    <= 134/|max| and |x| <= |max|): the slot is clamped as an unsigned
//    integer instead, which maps every NaN bit pattern (exponent all ones,
//    either sign) above 271, hence to the last pair, and the comparison
//    with NaN is false, so NaN again picks v15.
struct Iq4Lut {
    float v[16];
    float2 pair[272];  // (v[mu-1], v[mu]) by floor(x) + 136
    uint8_t cnt[272];  // mu - 1 by floor(x) + 136
};

__device__ __forceinline__ float iq4_clamp(float x) { return fmaxf(fminf(x, 127.0f), -128.0f); }
__device__ __forceinline__ int iq4_slot(float xc) {  // floor(xc) + 136 for xc in [-136, 136)
    return (int)__float_as_uint(__fadd_rd(xc, 12582912.0f)) - 0x4B400000 + 136;
}
__device__ __forceinline__ int iq4_slot_bounded(float x) {  // x in [-136, 136) or NaN
    return (int)min(__float_as_uint(__fadd_rd(x, 12582912.0f)) - (0x4B400000u - 136u), 271u);
}
__device__ __forceinline__ int best_index_iq4(const Iq4Lut &L, float x) {
    const float xc = iq4_clamp(x);
    const int f = iq4_slot(xc);
    const float2 p = L.pair[f];
    const int mu = 1 + L.cnt[f];
    return (xc - p.x < p.y - xc) ? mu - 1 : mu;
}
__device__ __forceinline__ int best_index_iq4_bounded(const Iq4Lut &L, float x) {
    const int f = iq4_slot_bounded(x);
    const float2 p = L.pair[f];
    const int mu = 1 + L.cnt[f];
    return (x - p.x < p.y - x) ? mu - 1 : mu;
}
// The codebook value best_index_iq4 selects, for x in [-136, 136) or NaN.
__device__ __forceinline__ float best_value_iq4_bounded(const Iq4Lut &L, float x) {
    const float2 p = L.pair[iq4_slot_bounded(x)];
    return (x - p.x < p.y - x) ? p.x : p.y;
}

__device__ void init_iq4_lut(Iq4Lut &L) {
    for (int i = threadIdx.x; i < 16; i += blockDim.x) L.v[i] = d_kv_f[i];
    for (int f = threadIdx.x; f < 272; f += blockDim.x) {
        int c = 0;
        for (int k = 1; k <= 14; k++) c += (d_kv_f[k] <= (float)(f - 136)) ? 1 : 0;
        L.cnt[f] = (uint8_t)c;
        L.pair[f] = make_float2(d_kv_f[c], d_kv_f[c + 1]);
    }
}

// ceil(t) for 0 <= t <= 2^22 as an int: RU(t + 2^23) is 2^23 + ceil(t),
// whose low mantissa bits are the result (no conversion instruction).
__device__ __forceinline__ int iq4_ceil(float t) {
    return (int)(__float_as_uint(__fadd_ru(t, 8388608.0f)) & 0x7FFFFFu);
}

// XS: a warp encodes one 256-element super-block (8 blocks of 32).
// NL: a warp encodes 8 consecutive 32-element blocks (each its own super-block).
// Each warp owns a contiguous, balanced range of units and walks it in
// batches of up to 32: the sequential sigma^2 folds of quant_iq.rs:1037 (256
// elements for XS, 32 per block for NL) run one unit per lane first, so each
// serial chain is issued once instead of on all 32 lanes; the batch's units
// are then encoded one after another.
//
// FUSE: the fused error table (fuse.cuh): warps 0-6 encode one unit each per
// stage (a batch of one), warp 7 folds.
template <bool XS, bool FUSE>
__global__ void __launch_bounds__(256, (!XS && !FUSE) ? 4 : 0) enc_iq4_kernel(EncArgs a) {  // plain NL: 4 blocks/SM measured 4 % faster
    __shared__ Iq4Lut lut;
    // block b's element pair p as (x[2p], x[2p+1], w[2p], w[2p+1]) at
    // s_xw[wid][b * 17 + p]: one 16-byte load per pair in the trial loop, the
    // blocks 17 slots apart so that lanes on different blocks use other banks
    __shared__ float4 s_xw[8][8 * 17];
    __shared__ float2 s_res[8][8][16];
    __shared__ float s_scale[8][8];
    __shared__ float s_sig[8][32][8];
    __shared__ float s_mx[8][8];
    __shared__ uint8_t s_job[8][128];
    __shared__ __align__(16) uint8_t s_out[8][144];
    __shared__ uint8_t s_l[8][256];
    init_iq4_lut(lut);
    __syncthreads();
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int b = lane >> 2, q = lane & 3;
    const int64_t ne0 = a.src.ne0;
    const int64_t nunits = XS ? a.n_rows * (ne0 >> 8) : (a.n_rows * (ne0 >> 5) + 7) >> 3;
    const int64_t bpr = ne0 >> 5;
    const int64_t nblk = a.n_rows * bpr;
    const int64_t nwarps = (int64_t)gridDim.x * 8, wg = (int64_t)blockIdx.x * 8 + wid;
    const int64_t u_lo = nunits * wg / nwarps, u_hi = nunits * (wg + 1) / nwarps;
    constexpr int NWE = 7;
    extern __shared__ __align__(16) uint8_t iq4_fuse_smem[];
    FuseSmem<NWE> *F = reinterpret_cast<FuseSmem<NWE> *>(iq4_fuse_smem);
    // IQ4_NL units: eight blocks, flat over the tensor (direct) or the eight
    // blocks from 256 u of row r at unit r * upr + u (fused, rows aligned)
    const int64_t upr = (bpr + 7) >> 3;
    auto unit_blk0 = [&](int64_t g) -> int64_t {
        if (!FUSE) return g * 8;
        const int64_t r = g / upr;
        return r * bpr + (g - r * upr) * 8;
    };
    auto unit_nb = [&](int64_t g) -> int {
        const int64_t left = FUSE ? bpr - (g - (g / upr) * upr) * 8 : nblk - g * 8;
        return (int)(left < 8 ? left : 8);
    };
    if constexpr (FUSE) {
        fuse_setup(*F);
        if (wid == NWE) {
            fuse_fold(*F, a, XS ? (ne0 >> 8) : upr, lane);
            return;
        }
    }
    auto units = [&](int64_t b0, int batch) {
    // sigma2 = 2 * (sequential sum of x^2 over the super-block) / size, one unit per lane
    {
        const int64_t gu = b0 + lane;
        if (lane < batch) {
            if (XS) {
                const int64_t nsb = ne0 >> 8;
                const int64_t row = gu / nsb, col = (gu - row * nsb) * 256;
                float s = 0.0f;
#pragma unroll 4
                for (int m = 0; m < 32; m++) {
                    float v[8];
                    load8(a.src, row, col + m * 8, v);
#pragma unroll
                    for (int k = 0; k < 8; k++) s += v[k] * v[k];
                }
                s_sig[wid][lane][0] = 2.0f * s / 256.0f;
            } else {
                const int64_t ub0 = unit_blk0(gu);
                const int unb = unit_nb(gu);
#pragma unroll 1
                for (int bb = 0; bb < unb; bb++) {
                    const int64_t blk = ub0 + bb;
                    const int64_t row = blk / bpr, col = (blk - row * bpr) * 32;
                    float s = 0.0f;
#pragma unroll
                    for (int m = 0; m < 4; m++) {
                        float v[8];
                        load8(a.src, row, col + m * 8, v);
#pragma unroll
                        for (int k = 0; k < 8; k++) s += v[k] * v[k];
                    }
                    s_sig[wid][lane][bb] = 2.0f * s / 32.0f;
                }
            }
        }
        __syncwarp();
    }
    for (int u = 0; u < batch; u++) {
        const int64_t g = b0 + u;
        // this lane group's 32-block: row and column
        int64_t row, col;
        bool valid = true;
        if (XS) {
            const int64_t nsb = ne0 >> 8;
            row = g / nsb;
            col = (g - row * nsb) * 256 + b * 32;
        } else {
            const int64_t blk = unit_blk0(g) + b;
            valid = b < unit_nb(g);
            row = valid ? blk / bpr : 0;
            col = valid ? (blk - row * bpr) * 32 : 0;
        }
        const float *imr = valid ? im_row(a.im, ne0, a.row0 + row * a.row_step) : nullptr;
        float v[8], base[8];
        if (valid) {
            load8(a.src, row, col + q * 8, v);
            if (imr) load_im8(imr, col + q * 8, base);
        } else {
#pragma unroll
            for (int k = 0; k < 8; k++) v[k] = 0.0f;
        }
        const float sig = s_sig[wid][u][XS ? 0 : b];
        {
            float wk[8];
#pragma unroll
            for (int k = 0; k < 8; k++) wk[k] = imr ? base[k] * sqrtf(sig + v[k] * v[k]) : v[k] * v[k];
            float4 *xw = &s_xw[wid][b * 17 + q * 4];
#pragma unroll
            for (int p = 0; p < 4; p++) xw[p] = make_float4(v[2 * p], v[2 * p + 1], wk[2 * p], wk[2 * p + 1]);
        }
        __syncwarp();
        // max |x| of the block, first strict maximum (quant_iq.rs:1053-1059):
        // each of the block's four lanes scans its own eight elements, then
        // a butterfly keeps the lower lane's value unless the higher lane's is
        // strictly larger, which is the serial scan's first-maximum rule.
        float amax = 0.0f, mx = 0.0f;
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const float av = fabsf(v[k]);
            if (av > amax) { amax = av; mx = v[k]; }
        }
#pragma unroll
        for (int off = 1; off <= 2; off <<= 1) {
            const float oa = __shfl_xor_sync(0xffffffffu, amax, off), om = __shfl_xor_sync(0xffffffffu, mx, off);
            if ((q & off) == 0 ? oa > amax : !(amax > oa)) { amax = oa; mx = om; }
        }
        const bool live = !(amax < kGroupMaxEps);
        // Trials whose code vector repeats the previous trial's are skipped.
        // For jobs 1..15, id_j = (j - 135)/max moves monotonically with j, so
        // each element's code (a monotone step function of id*x) changes
        // only where id_j*x crosses a decision point between neighbouring
        // codebook values: (j - 135) x/max = T at j* = 135 + T max/x.  A
        // repeated trial has the same (sumqx, sumq2) as the one before it
        // and leaves the selection chain's state as it is, accepted or not.
        // The codes at trials 1 and 15 (exact) count the crossings (at most
        // two: the span of id*x is 14 |x|/|max|, the codebook steps are >= 11);
        // j* is known to well within 0.01 (rounding of id, of the product and
        // of the decision, and of the estimate, for |x| >= |max|/30 as any
        // crossing needs), so the grids ceil(j* -+ 0.01) are marked.
        unsigned int jmask = 0;
        if (live) {
            if (fabsf(mx) < INFINITY) {
                const float id1 = (-7.0f + -127.0f) / mx, id15 = (7.0f + -127.0f) / mx;
#pragma unroll
                for (int k = 0; k < 8; k++) {
                    const int i1 = best_index_iq4_bounded(lut, id1 * v[k]), i15 = best_index_iq4_bounded(lut, id15 * v[k]);
                    if (i1 != i15) {
                        const float r = mx / v[k];
                        const int lo = min(i1, i15), hi = max(i1, i15);
#pragma unroll
                        for (int c = 0; c < 2; c++) {
                            if (lo + c < hi) {
                                const float T = (lut.v[lo + c] + lut.v[lo + c + 1]) * 0.5f;
                                const float js = 135.0f + T * r;
                                jmask |= 1u << iq4_ceil(fminf(fmaxf(js - 0.01f, 2.0f), 15.0f));
                                jmask |= 1u << iq4_ceil(fminf(fmaxf(js + 0.01f, 2.0f), 15.0f));
                            }
                        }
                    }
                }
            } else {
                jmask = 0xFFFFu;
            }
            jmask |= 3u;  // the initial grid and trial 1
        }
        jmask |= __shfl_xor_sync(0xffffffffu, jmask, 1);
        jmask |= __shfl_xor_sync(0xffffffffu, jmask, 2);
        // (block, job) list of the unit, dealt to the warp's 32 lanes; lane q
        // of a block lists the jobs among bits [4q, 4q + 4)
        {
            const int cnt = __popc(jmask);
            int incl = q == 0 ? cnt : 0;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int t = __shfl_up_sync(0xffffffffu, incl, off);
                if (lane >= off) incl += t;
            }
            const int njobs = __shfl_sync(0xffffffffu, incl, 31);
            int pos = __shfl_sync(0xffffffffu, incl, lane - q) - cnt + __popc(jmask & ((1u << (4 * q)) - 1u));
            unsigned int bits = (jmask >> (4 * q)) & 0xFu;
            while (bits != 0) {
                s_job[wid][pos++] = (uint8_t)((b << 4) | (4 * q + __ffs(bits) - 1));
                bits &= bits - 1;
            }
            if (q == 0) s_mx[wid][b] = mx;
            __syncwarp();
            // job 0: the initial grid d = -max/v0; jobs 1..15: itry = job - 8
            for (int t = lane; t < njobs; t += 32) {
                const int code = s_job[wid][t];
                const int jb = code >> 4, j = code & 15;
                const float jmx = s_mx[wid][jb];
                const float4 *jxw = &s_xw[wid][jb * 17];
                const float id = j == 0 ? 1.0f / (-jmx / -127.0f) : ((float)(j - 8) + -127.0f) / jmx;
                float sumqx = 0.0f, sumq2 = 0.0f;
#pragma unroll
                for (int p = 0; p < 16; p++) {  // element pairs; products feed scalar sums only
                    const float4 f = jxw[p];
                    const float2 xi = make_float2(f.x, f.y);
                    const float2 y = __fmul2_rn(make_float2(id, id), xi);
                    const float2 qv = make_float2(best_value_iq4_bounded(lut, y.x), best_value_iq4_bounded(lut, y.y));
                    const float2 wq = __fmul2_rn(make_float2(f.z, f.w), qv);
                    const float2 sx = __fmul2_rn(wq, xi);
                    const float2 s2 = __fmul2_rn(wq, qv);
                    sumqx = __fadd_rn(sumqx, sx.x);
                    sumq2 = __fadd_rn(sumq2, s2.x);
                    sumqx = __fadd_rn(sumqx, sx.y);
                    sumq2 = __fadd_rn(sumq2, s2.y);
                }
                s_res[wid][jb][j] = make_float2(sumqx, sumq2);
            }
        }
        __syncwarp();
        if (q == 0) {
            float d = 0.0f;
            if (live) {
                const float2 r0 = s_res[wid][b][0];
                d = r0.y > 0.0f ? r0.x / r0.y : 0.0f;
                float best = d * r0.x;
                unsigned int m = jmask & ~1u;  // evaluated trials, in order
                while (m != 0) {
                    const int j = __ffs(m) - 1;
                    m &= m - 1;
                    const float2 r = s_res[wid][b][j];
                    if (r.y > 0.0f && r.x * r.x > best * r.y) {
                        d = r.x / r.y;
                        best = d * r.x;
                    }
                }
            }
            s_scale[wid][b] = d;
        }
        __syncwarp();
        uint8_t *o = s_out[wid];
        float idl;
        if (XS) {
            // largest |scale| of the eight blocks, first strict maximum
            // (quant_iq.rs:1094-1097), by a butterfly over the blocks' lanes
            float amax_s = 0.0f, max_s = 0.0f;
            {
                const float dv = s_scale[wid][b];
                if (fabsf(dv) > 0.0f) { amax_s = fabsf(dv); max_s = dv; }
            }
#pragma unroll
            for (int off = 4; off <= 16; off <<= 1) {
                const float oa = __shfl_xor_sync(0xffffffffu, amax_s, off), om = __shfl_xor_sync(0xffffffffu, max_s, off);
                if ((lane & off) == 0 ? oa > amax_s : !(amax_s > oa)) { amax_s = oa; max_s = om; }
            }
            const float d = -max_s / 32.0f;
            const float id = d != 0.0f ? 1.0f / d : 0.0f;
            const int l = clampi(nearest_int(id * s_scale[wid][b]), -32, 31);
            const float dl = d * (float)l;
            idl = dl != 0.0f ? 1.0f / dl : 0.0f;
            if (lane == 0) {
                const uint16_t h = f16_bits(d);
                o[0] = (uint8_t)(h & 0xFF);
                o[1] = (uint8_t)(h >> 8);
            }
            // scales_h (2 B) and scales_l (4 B) from the eight 6-bit scales
            const int lu = l + 32;
            int lus[8];
#pragma unroll
            for (int bb = 0; bb < 8; bb++) lus[bb] = __shfl_sync(0xffffffffu, lu, bb * 4);
            if (lane == 0) {
                uint16_t h16 = 0;
#pragma unroll
                for (int bb = 0; bb < 8; bb++) h16 |= (uint16_t)(((lus[bb] >> 4) & 3) << (2 * bb));
                o[2] = (uint8_t)(h16 & 0xFF);
                o[3] = (uint8_t)(h16 >> 8);
#pragma unroll
                for (int t = 0; t < 4; t++) o[4 + t] = (uint8_t)((lus[2 * t] & 0xF) | ((lus[2 * t + 1] & 0xF) << 4));
            }
        } else {
            const float sc = s_scale[wid][b];
            idl = sc != 0.0f ? 1.0f / sc : 0.0f;
            if (q == 0) {
                const uint16_t h = f16_bits(sc);
                o[b * 18] = (uint8_t)(h & 0xFF);
                o[b * 18 + 1] = (uint8_t)(h >> 8);
            }
        }
#pragma unroll
        for (int k = 0; k < 8; k++) s_l[wid][lane * 8 + k] = (uint8_t)best_index_iq4(lut, idl * v[k]);
        __syncwarp();
        // q4[16*i + j] = L[32i + j] | L[32i + 16 + j] << 4; lane packs 4 bytes of its block
        {
            const uint8_t *L = s_l[wid] + b * 32;
            uint8_t *qo = XS ? o + 8 + b * 16 : o + b * 18 + 2;
#pragma unroll
            for (int t = 0; t < 4; t++) {
                const int jj = q * 4 + t;
                qo[jj] = (uint8_t)(L[jj] | (L[16 + jj] << 4));
            }
        }
        __syncwarp();
        if (FUSE) {
        } else if (XS) {
            const int64_t nsb = ne0 >> 8;
            const int64_t sbi = g - (g / nsb) * nsb;
            store_block(a.dst + (g / nsb) * a.dst_row_bytes + sbi * 136, o, 136, a.dst_aligned16 != 0, lane);
        } else {
            const int64_t blk0 = g * 8;
            const int nb = (int)(nblk - blk0 < 8 ? nblk - blk0 : 8);
            store_block(a.dst + blk0 * 18, o, nb * 18, a.dst_aligned16 && nb == 8, lane);
        }
        __syncwarp();
    }
    };
    if constexpr (!FUSE) {
        for (int64_t b0 = u_lo; b0 < u_hi; b0 += 32) units(b0, (int)(u_hi - b0 < 32 ? u_hi - b0 : 32));
    } else {
        const int64_t upr_f = XS ? (ne0 >> 8) : upr;
        FuseIter<NWE> it(a, upr_f, wid);
        uint32_t fk = 0;
        while (it.next()) {
            if (it.valid) units(it.row * upr_f + it.unit, 1);
            fuse_emit<XS ? SHC_TYPE_IQ4_XS : SHC_TYPE_IQ4_NL, XS ? 0 : 18>(*F, wid, fk, it.valid, a, it.row, it.unit,
                                                                          s_out[wid], lane);
        }
    }
}

}  // namespace shc

namespace shc {

// ---------------------------------------------------------------------------
// IQ2_XXS / IQ2_XS / IQ2_S / IQ3_XXS / IQ3_S (quant_iq.rs:275-935)
// ---------------------------------------------------------------------------
// V: 0 IQ2_XXS, 1 IQ2_XS, 2 IQ2_S, 3 IQ3_XXS, 4 IQ3_S (also the table slot).
template <int V>
struct IqCfg {
    static constexpr bool IQ2 = V < 3;
    static constexpr int BS = (V == 1 || V == 2) ? 16 : 32;  // block size
    static constexpr int NB = 256 / BS;                      // blocks per super-block
    static constexpr int G = IQ2 ? 8 : 4;                    // lattice dimension
    static constexpr int NG = BS / G;                        // lattice groups per block
    static constexpr int NSG = BS / 8;                       // sign groups per block
    static constexpr int KM = IQ2 ? 3 : 8;                   // k_max_q
    static constexpr int BITS = IQ2 ? 2 : 3;
    static constexpr int NT = V == 0 ? 13 : (V == 3 ? 31 : 19);
    static constexpr int IS_LO = V == 0 ? -6 : (V == 3 ? -15 : -9);
    static constexpr float STEP = IQ2 ? 0.1f : 0.2f;
    static constexpr bool PARITY = (V == 0 || V == 1 || V == 3);  // 7 stored sign bits + parity
    static constexpr bool QP = V == 0;                            // make_qp_quants seed
    static constexpr bool SIG2X = (V >= 2);                       // sigma2 = 2 * mean(x^2)
    static constexpr int OUT = V == 0 ? 66 : V == 1 ? 74 : V == 2 ? 82 : V == 3 ? 98 : 110;
    static constexpr int KMAP = IQ2 ? 6561 : 4096;
};

// Levels of one block packed BITS per element, group k (G levels, the
// lattice index's own bit layout) at bit k*G*BITS; groups never straddle
// the two words (IQ2: 4 groups of 16 bits per word, IQ3: 5 of 12).
template <int V>
struct Levels {
    using C = IqCfg<V>;
    static constexpr int GB = C::G * C::BITS;
    static constexpr int GPW = 64 / GB;
    uint64_t p0 = 0, p1 = 0;
    __device__ __forceinline__ void set_group(int k, uint32_t g) {
        const uint64_t mask = (1ull << GB) - 1;
        if (k < GPW) {
            const int sh = k * GB;
            p0 = (p0 & ~(mask << sh)) | ((uint64_t)g << sh);
        } else {
            const int sh = (k - GPW) * GB;
            p1 = (p1 & ~(mask << sh)) | ((uint64_t)g << sh);
        }
    }
    __device__ __forceinline__ uint32_t group(int k) const {
        const uint64_t mask = (1ull << GB) - 1;
        return k < GPW ? (uint32_t)((p0 >> (k * GB)) & mask) : (uint32_t)((p1 >> ((k - GPW) * GB)) & mask);
    }
    __device__ __forceinline__ int level(int i) const {  // i compile-time after unrolling
        const int k = i / C::G, w = i % C::G;
        const int sh = (k % GPW) * GB + w * C::BITS;
        return (int)(((k < GPW ? p0 : p1) >> sh) & ((1u << C::BITS) - 1));
    }
};

// Compact kmap index of a group given in the lattice bit layout.
template <int V>
__device__ __forceinline__ int kmap_index(uint32_t g) {
    using C = IqCfg<V>;
    if (!C::IQ2) return (int)g;  // IQ3: sum l_i << 3i is already the index
    int u = 0;
#pragma unroll
    for (int i = C::G - 1; i >= 0; i--) u = u * 3 + (int)((g >> (2 * i)) & 3u);
    return u;
}

// Round one group to the lattice at `id` (quant_iq.rs: l = clamp(round(
// 0.5*(id*x - 1)), 0, kmax-1)); returns the group's packed levels.
template <int V>
__device__ __forceinline__ uint32_t round_group(const float *xg, float id) {
    using C = IqCfg<V>;
    uint32_t g = 0;
#pragma unroll
    for (int i = 0; i < C::G; i++) {
        const int l = round_clamp0_i(0.5f * (id * xg[i] - 1.0f), (float)(C::KM - 1));
        g |= (uint32_t)l << (C::BITS * i);
    }
    return g;
}

// Weighted sums of a block for packed levels: sumqx += w*x*q, sumq2 += w*q*q.
template <int V>
__device__ __forceinline__ void block_sums(const float *xv, const float *w, const Levels<V> &lv, float &sx, float &s2) {
    using C = IqCfg<V>;
    float a = 0.0f, c = 0.0f;
#pragma unroll
    for (int i = 0; i < C::BS; i++) {
        const float q = odd_level((uint32_t)lv.level(i));
        a += w[i] * xv[i] * q;
        c += w[i] * q * q;
    }
    sx = a;
    s2 = c;
}

// nearest_int for the make_qp_quants values: f32::round half away from zero
// with three adds, and the integer read from the mantissa of r + 1.5*2^23,
// exact for |r| < 2^22; NaN and larger magnitudes take the general path.
__device__ __forceinline__ int nearest_int_qp(float y) {
    if (!(fabsf(y) < 4194304.0f)) return nearest_int(y);
    return (int)__float_as_uint(__fadd_rn(round_away_small(y), 12582912.0f)) - 0x4B400000;
}

// make_qp_quants (quant_iq.rs:170-241), n = 32, nmax = 4: the IQ2_XXS seed,
// computed by the four lanes 4b..4b+3 of block b (u = lane & 3).  The max
// fold is order-independent (NaN-ignoring, from +0) and is split over the
// four lanes; the nine candidate scales' errors (each a serial sum over the
// block, as in the reference) are split over the lanes as well; the choice
// among them (first strict minimum), the final levels and the coordinate
// descent are sequential and run on lane u == 0, with the levels `ls` in
// shared memory.  Every lane of the warp must call it.
__device__ float make_qp_quants32_x4(const float *x, const float *w, uint8_t *ls, int lane) {
    constexpr int n = 32, nmax = 4;
    const int u = lane & 3, grp = lane & ~3;
    float max = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) max = rmaxf(max, x[u * 8 + i]);
    max = rmaxf(max, __shfl_xor_sync(0xffffffffu, max, 1));
    max = rmaxf(max, __shfl_xor_sync(0xffffffffu, max, 2));
    const bool dead = max < kGroupMaxEps;
    // trial t: 0 the initial iscale (levels wrap as u8, no clamp), 1..8 is = -4..-1, 1..4
    auto iscale_of = [&](int t) -> float {
        if (t == 0) return (float)nmax / max;
        const int is = t <= 4 ? t - 5 : t - 4;
        return (0.1f * (float)is + (float)nmax) / max;
    };
    float mine[3];
#pragma unroll
    for (int r = 0; r < 3; r++) {
        const int t = u + 4 * r;
        float mse = 0.0f;
        if (!dead && t < 9) {
            const float isc = iscale_of(t);
            const float scale = 1.0f / isc;
            for (int i = 0; i < n; i++) {
                const int l = t == 0 ? (int)(uint8_t)nearest_int_qp(isc * x[i]) : min(nearest_int_qp(isc * x[i]), nmax);
                const float diff = x[i] - scale * (float)l;
                mse += w[i] * diff * diff;
            }
        }
        mine[r] = mse;
    }
    float best = 0.0f, iscale = 0.0f;
#pragma unroll
    for (int t = 0; t < 9; t++) {
        const float mse = __shfl_sync(0xffffffffu, mine[t >> 2], grp | (t & 3));
        if (t == 0) {
            best = mse;
            iscale = iscale_of(0);
        } else if (mse < best) {
            best = mse;
            iscale = iscale_of(t);
        }
    }
    float res = 0.0f;
    if (!dead && u == 0) {
        float sumlx = 0.0f, suml2 = 0.0f;
        for (int i = 0; i < n; i++) {
            // l may be negative (the parity-flipped element): the sums take the
            // i32 value, the level buffer its u8 wrap, as the reference does
            const int l = min(nearest_int_qp(iscale * x[i]), nmax);
            ls[i] = (uint8_t)l;
            sumlx += w[i] * x[i] * (float)l;
            suml2 += w[i] * (float)(l * l);
        }
        for (int it = 0; it < 5; it++) {
            int n_changed = 0;
#pragma unroll 1
            for (int i = 0; i < n; i++) {
                const float wi = w[i];
                const float li = (float)ls[i];
                const float slx = sumlx - wi * x[i] * li;
                const float sl2 = suml2 - wi * li * li;
                if (slx > 0.0f && sl2 > 0.0f) {
                    const int new_l = min(nearest_int_qp(x[i] * sl2 / slx), nmax);
                    if ((uint8_t)new_l != ls[i]) {
                        const float slx2 = slx + wi * x[i] * (float)new_l;
                        const float sl22 = sl2 + wi * (float)(new_l * new_l);
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
        res = suml2 > 0.0f ? sumlx / suml2 : 0.0f;
    }
    return res;
}

// An off-grid kmap entry m < 0 holds -(1 + first entry + (count << kListCountShift)).
constexpr int kListCountShift = 19;

// Neighbour search layout per variant.  IQ2 lists (8 dimensions, ~10-60
// entries) are scanned cooperatively: a chunk of CJ jobs queues its off-grid
// groups as tasks, and rounds of 32 tasks share the warp with equal
// candidate ranges per lane, scored from per-task term tables.  IQ3 lists (4
// dimensions, ~10 entries) are scanned by the lane that owns the job, from
// lists staged in shared memory, four candidates per step, with 16 warps per
// block (measured: a cooperative scan issued fewer instructions for IQ3 but
// stalled more and ran slower).
template <int V>
struct IqSearch {
    static constexpr bool COOP = V < 3;
    static constexpr int CJ = 32;                  // jobs per chunk (COOP)
    static constexpr bool LISTS_SMEM = !COOP;      // IQ3: 40-50 KB of lists
    static constexpr int WARPS = COOP ? 8 : 16;    // warps per block
};

// Per-warp shared state; block arrays padded to BS+1 so lanes working on
// different blocks hit different banks.
template <int V>
struct IqWarpSmem {
    using C = IqCfg<V>;
    static constexpr bool COOP = IqSearch<V>::COOP;
    static constexpr int BP = C::BS + 1;
    static constexpr int MAXT = COOP ? IqSearch<V>::CJ * C::NG : 1;  // search tasks per chunk of jobs
    static constexpr int TS = C::G * C::KM;      // terms waux_i*diff*diff per round slot
    uint32_t key[MAXT];                          // task: winning packed levels, or ~0u
    unsigned long long rkey[COOP ? 32 : 1];      // round slot: best (d2 bits, (position, levels))
    union {
        float x[256];                            // the super-block (weights and sigma^2 only)
        // term (i, l) of round slot t at [(i*KM + l)*32 + t]: a slot's terms
        // share one bank, so lanes scanning different lists never collide
        float tab[COOP ? 32 * TS : 1];
    };
    float xv[C::NB * BP];
    float w[C::NB * BP];
    float wa[C::NB * BP];
    float2 jres[C::NB * C::NT];                  // (sumqx, sumq2) of every (block, trial) job
    int pre[COOP ? 33 : 1];                      // round slot: first group of four in the flattened lists
    int rbase[COOP ? 32 : 1];                    // round slot: list offset
    int tq_m[MAXT];                              // task: kmap entry (< 0: neighbour list offset)
    float tq_s[MAXT];                            // task: scale the candidates are scored at
    uint16_t tq_x[MAXT];                         // task: offset of the group in xv / wa
    float bscale0[C::NB];                        // chain start scale per block (qp seed or max/(2k-1))
    float bmax[C::NB];                           // max |x| (or the qp effective max) per block
    float bscale[C::NB];                         // final block scale
    uint8_t live[C::NB];
    uint8_t signs[32];                           // per 8-element sign group
    float sigb[32];                              // sigma^2 of the warp's next 32 super-blocks
    uint8_t qpl[C::QP ? 256 : 1];                // make_qp_quants levels per block (IQ2_XXS)
    float qps[C::QP ? C::NB : 1];                // make_qp_quants result per block (IQ2_XXS)
    uint16_t gidx[64];                           // grid index per lattice group
    // IQ3: per-block rounding requests served one (block, group) per lane
    float rid[COOP ? 1 : C::NB];                 // id the block's groups round at
    float rsc[COOP ? 1 : C::NB];                 // scale their neighbours are scored at
    uint32_t rtodo[COOP ? 1 : C::NB];            // groups to round (0: none)
    uint16_t rg[COOP ? 1 : C::NB * C::NG];       // result: the group's packed levels
    uint8_t roff[COOP ? 1 : C::NB * C::NG];      // result: 1 if it was off the grid
    __align__(16) uint8_t out[112];
};

// Exclusive prefix of `cnt` over the warp; returns the lane's offset and
// the total in `total`.
__device__ __forceinline__ int warp_exclusive_scan(int cnt, int lane, int &total) {
    int pos = cnt;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, pos, d);
        if (lane >= d) pos += o;
    }
    total = __shfl_sync(0xffffffffu, pos, 31);
    return pos - cnt;
}

// find_best_neighbour (quant_iq.rs:137-167).  The reference keeps the first
// candidate whose d2 = sum_i waux_i*(scale*g_i - x_i)^2 (a serial sum over
// the lattice dimension) is strictly below the running best, which starts at
// f32::MAX: the candidate with the smallest (d2, list position) among those
// with d2 < f32::MAX.  d2 >= +0, so its bits order like its value and
// (bits << 32 | position) is one 64-bit key.

// Per-lane scan of one list (IQ3): returns the winner's packed levels, or ~0u.
// m is the group's kmap entry (first entry and length of its list); the
// entries start on a four-entry boundary and are padded to a multiple of
// four with copies of the last entry, so each 64-bit load brings four
// candidates whose distances are independent chains.  Kept out of line: its
// callers are unrolled over the groups.
template <int V>
__device__ __noinline__ uint32_t lane_search(const uint16_t *l16, int m, const float *xg, const float *wg,
                                                float scale) {
    using C = IqCfg<V>;
    constexpr uint32_t MASK = (1u << C::BITS) - 1;
    const uint32_t v = (uint32_t)(-m - 1);
    const int n = (int)(v >> kListCountShift);
    const uint2 *q4 = reinterpret_cast<const uint2 *>(l16 + (v & ((1u << kListCountShift) - 1)));
    float xi[C::G], wi[C::G];
#pragma unroll
    for (int i = 0; i < C::G; i++) {
        xi[i] = xg[i];
        wi[i] = wg[i];
    }
    float best = FLT_MAX;
    uint32_t bc = ~0u;
    for (int g = 0; g < (n + 3) >> 2; g++) {
        const uint2 w4 = q4[g];
        const uint32_t cc[4] = {w4.x & 0xFFFFu, w4.x >> 16, w4.y & 0xFFFFu, w4.y >> 16};
        float d2[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int i = 0; i < C::G; i++)
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const float diff = scale * odd_level((cc[u] >> (C::BITS * i)) & MASK) - xi[i];
                d2[u] += wi[i] * diff * diff;
            }
#pragma unroll
        for (int u = 0; u < 4; u++)
            if (d2[u] < best) {  // in list order: strict keeps the first
                best = d2[u];
                bc = cc[u];
            }
    }
    return bc;
}

// Cooperative scan of the queued tasks [0, T) (IQ2), 32 per round: each lane
// tabulates one task's terms per (dimension, level); the round's lists are then laid end to end in groups of four entries (each list
// padded with copies of its last entry) and cut into 32 equal contiguous
// ranges of groups, one per lane, so every lane scores the same number of
// candidates whatever the lists' lengths.  A group is one 32- or 64-bit load
// and four independent distance chains.  A lane keeps the first minimum of
// its part of each list and merges it into that list's key (shared-memory
// atomicMin on (d2 bits, position)); only neighbouring lanes ever share a
// list.  On return key[q] holds task q's winning packed levels, or ~0u.
// d2 = sum_i waux_i*(scale*g_i - x_i)^2 in the reference's order
// (quant_iq.rs:152-156), from 0, one dimension after another.
template <int V>
__device__ __noinline__ void search_tasks(IqWarpSmem<V> &S, int T, const void *lists, const uint16_t *gco, int lane) {
    using C = IqCfg<V>;
    constexpr int KM = C::KM, G = C::G;
    constexpr uint32_t MASK = (1u << C::BITS) - 1;
    const uint8_t *l8 = static_cast<const uint8_t *>(lists);
    const uint16_t *l16 = static_cast<const uint16_t *>(lists);
    for (int r0 = 0; r0 < T; r0 += 32) {
        const int q = r0 + lane;
        int ng = 0;
        if (q < T) {
            // the kmap entry holds the list's first entry (a multiple of 4) and length
            const uint32_t v = (uint32_t)(-S.tq_m[q] - 1);
            ng = (int)((v >> kListCountShift) + 3) >> 2;
            S.rbase[lane] = (int)(v & ((1u << kListCountShift) - 1));
            const float scale = S.tq_s[q];
            const int xo = S.tq_x[q];
            float *tb = S.tab + lane;
#pragma unroll
            for (int i = 0; i < G; i++) {
                const float xi = S.xv[xo + i], wi = S.wa[xo + i];
#pragma unroll
                for (int l = 0; l < KM; l++) {
                    const float diff = scale * (float)(2 * l + 1) - xi;
                    tb[(i * KM + l) * 32] = wi * diff * diff;
                }
            }
        }
        S.rkey[lane] = ~0ull;
        int tot;
        S.pre[lane] = warp_exclusive_scan(ng, lane, tot);  // in groups of four entries
        if (lane == 0) S.pre[32] = tot;
        __syncwarp();
        const int g0 = (int)(((int64_t)tot * lane) >> 5), g1 = (int)(((int64_t)tot * (lane + 1)) >> 5);
        if (g0 < g1) {
            int t = 0;  // the slot holding group g0: smallest t with pre[t+1] > g0
            for (int hi = 31; t < hi;) {
                const int mid = (t + hi) >> 1;
                if (S.pre[mid + 1] > g0) hi = mid;
                else t = mid + 1;
            }
            int end = S.pre[t + 1];
            int ent = S.rbase[t] - 4 * S.pre[t];  // slot t's group g sits at entry ent + 4*g
            const float *tb = S.tab + t;
            uint32_t bh = 0xFFFFFFFFu, bl = 0xFFFFFFFFu;
            for (int g = g0; g < g1; g++) {
                if (g == end) {  // this lane's part of slot t is done: merge, move to the next nonempty slot
                    if (bh != 0xFFFFFFFFu) atomicMin(&S.rkey[t], ((unsigned long long)bh << 32) | bl);
                    bh = bl = 0xFFFFFFFFu;
                    do {
                        t++;
                    } while (S.pre[t + 1] <= g);
                    end = S.pre[t + 1];
                    ent = S.rbase[t] - 4 * S.pre[t];
                    tb = S.tab + t;
                }
                uint32_t cc[4];
                if (V == 0) {
                    const uint32_t w4 = __ldg(reinterpret_cast<const uint32_t *>(l8 + ent + 4 * g));
#pragma unroll
                    for (int u = 0; u < 4; u++) cc[u] = gco[(w4 >> (8 * u)) & 255u];
                } else {
                    const uint2 w4 = __ldg(reinterpret_cast<const uint2 *>(l16 + ent + 4 * g));
                    cc[0] = w4.x & 0xFFFFu;
                    cc[1] = w4.x >> 16;
                    cc[2] = w4.y & 0xFFFFu;
                    cc[3] = w4.y >> 16;
                }
                float d2[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                for (int i = 0; i < G; i++)
#pragma unroll
                    for (int u = 0; u < 4; u++) d2[u] += tb[(i * KM + ((cc[u] >> (C::BITS * i)) & MASK)) * 32];
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const uint32_t kh = __float_as_uint(d2[u]);
                    if (d2[u] < FLT_MAX && kh < bh) {  // positions rise within the lane: strict keeps the first
                        bh = kh;
                        bl = ((uint32_t)(4 * g + u) << 16) | cc[u];  // (position, the candidate's levels)
                    }
                }
            }
            if (bh != 0xFFFFFFFFu) atomicMin(&S.rkey[t], ((unsigned long long)bh << 32) | bl);
        }
        __syncwarp();
        if (q < T) {
            const unsigned long long kk = S.rkey[lane];
            S.key[q] = kk == ~0ull ? 0xFFFFFFFFu : (uint32_t)kk & 0xFFFFu;
        }
        __syncwarp();
    }
}

// Round the groups `todo` of one block at `id` (the trial loops of
// quant_iq.rs): on-grid groups go into lv.  Off-grid groups are searched
// here at `scale` (IQ3, per lane) or leave their kmap entry in mk for the
// cooperative search (IQ2).  Returns the off-grid mask.
template <int V>
__device__ __forceinline__ uint32_t round_block(IqWarpSmem<V> &S, const int *kmap, const uint16_t *l16, int xb,
                                                float id, float scale, uint32_t todo, Levels<V> &lv,
                                                int (&mk)[IqCfg<V>::NG], int *status) {
    using C = IqCfg<V>;
    uint32_t offm = 0;
    if (IqSearch<V>::COOP) {
#pragma unroll
        for (int k = 0; k < C::NG; k++) {
            mk[k] = 0;
            if (!((todo >> k) & 1u)) continue;
            const uint32_t g = round_group<V>(S.xv + xb + k * C::G, id);
            const int m = kmap[kmap_index<V>(g)];
            if (m >= 0) {
                lv.set_group(k, g);
            } else {
                offm |= 1u << k;
                mk[k] = m;
            }
        }
    } else {
#pragma unroll 1
        for (int k = 0; k < C::NG; k++) {
            if (!((todo >> k) & 1u)) continue;
            uint32_t g = round_group<V>(S.xv + xb + k * C::G, id);
            const int m = kmap[kmap_index<V>(g)];
            if (m < 0) {
                offm |= 1u << k;
                g = lane_search<V>(l16, m, S.xv + xb + k * C::G, S.wa + xb + k * C::G, scale);
                if (g == ~0u) {
                    set_status(status, SHC_ENONEIGHBOUR);
                    g = 0;
                }
            }
            lv.set_group(k, g);
        }
    }
    return offm;
}

// IQ2_XXS takes round_block out of line: its kernel is large enough that
// the three inlined copies cost more in instruction fetch than the calls.
template <int V>
__device__ __noinline__ uint32_t round_block_call(IqWarpSmem<V> &S, const int *kmap, const uint16_t *l16, int xb,
                                                  float id, float scale, uint32_t todo, Levels<V> &lv,
                                                  int (&mk)[IqCfg<V>::NG], int *status) {
    return round_block<V>(S, kmap, l16, xb, id, scale, todo, lv, mk, status);
}
template <int V>
__device__ __forceinline__ uint32_t round_block_sel(IqWarpSmem<V> &S, const int *kmap, const uint16_t *l16, int xb,
                                                    float id, float scale, uint32_t todo, Levels<V> &lv,
                                                    int (&mk)[IqCfg<V>::NG], int *status) {
    if constexpr (V == 0) return round_block_call<V>(S, kmap, l16, xb, id, scale, todo, lv, mk, status);
    else return round_block<V>(S, kmap, l16, xb, id, scale, todo, lv, mk, status);
}

// IQ3: round the groups S.rtodo[b] of every block b at S.rid[b], one
// (block, group) per lane, searching off-grid groups' neighbour lists at
// S.rsc[b]; results in S.rg / S.roff.  The same per-group steps as
// round_block, which walks a block's groups on one lane.  Every lane of the
// warp must call it.
template <int V>
__device__ __forceinline__ void round_groups_lanes(IqWarpSmem<V> &S, const int *kmap, const uint16_t *l16, int lane,
                                                   int *status) {
    using C = IqCfg<V>;
    constexpr int BP = C::BS + 1;
    __syncwarp();
#pragma unroll 1
    for (int task = lane; task < C::NB * C::NG; task += 32) {
        const int b = task / C::NG, k = task - b * C::NG;
        if (!((S.rtodo[b] >> k) & 1u)) continue;
        const int xo = b * BP + k * C::G;
        uint32_t g = round_group<V>(S.xv + xo, S.rid[b]);
        const int m = kmap[kmap_index<V>(g)];
        uint8_t off = 0;
        if (m < 0) {
            off = 1;
            g = lane_search<V>(l16, m, S.xv + xo, S.wa + xo, S.rsc[b]);
            if (g == ~0u) {
                set_status(status, SHC_ENONEIGHBOUR);
                g = 0;
            }
        }
        S.rg[task] = (uint16_t)g;
        S.roff[task] = off;
    }
    __syncwarp();
}

template <int V>
__device__ __forceinline__ void queue_tasks(IqWarpSmem<V> &S, int pos, uint32_t offm, const int (&mk)[IqCfg<V>::NG],
                                            int xb, float scale) {
    using C = IqCfg<V>;
#pragma unroll
    for (int k = 0; k < C::NG; k++) {
        if (!((offm >> k) & 1u)) continue;
        S.tq_m[pos] = mk[k];
        S.tq_s[pos] = scale;
        S.tq_x[pos] = (uint16_t)(xb + k * C::G);
        pos++;
    }
}

template <int V>
__device__ __forceinline__ void take_results(IqWarpSmem<V> &S, int pos, uint32_t offm, Levels<V> &lv, int *status) {
    using C = IqCfg<V>;
#pragma unroll
    for (int k = 0; k < C::NG; k++) {
        if (!((offm >> k) & 1u)) continue;
        uint32_t c = (uint32_t)S.key[pos++];
        if (c == ~0u) {
            set_status(status, SHC_ENONEIGHBOUR);
            c = 0;
        }
        lv.set_group(k, c);
    }
}

// FUSE: the fused error table (fuse.cuh): the last warp folds, the others
// encode; its slots take the fold warp's workspace when they fit there, else
// they follow the lists.
// Fused launches use 16 warps for every variant (one resident block per SM).
template <int V, bool FUSE>
struct IqWarps {
    static constexpr int value = FUSE ? 16 : IqSearch<V>::WARPS;
};

template <int V, bool FUSE>
__global__ void __launch_bounds__(IqWarps<V, FUSE>::value * 32, (IqSearch<V>::COOP && !FUSE) ? 2 : 1)
    enc_iq_lattice_kernel(EncArgs a, const int32_t *__restrict__ g_kmap, const void *__restrict__ g_lists,
                          int lists_bytes, const uint32_t *__restrict__ g_coords) {
    using C = IqCfg<V>;
    constexpr int BP = C::BS + 1;
    constexpr int NJ = C::NB * C::NT;
    constexpr int NW = IqWarps<V, FUSE>::value;
    constexpr bool COOP = IqSearch<V>::COOP;
    extern __shared__ __align__(16) uint8_t smem_raw[];
    // shared memory: compact kmap | grid coords (IQ2_XXS) | per-warp state |
    // neighbour lists (IQ3; IQ2 reads its lists through L1/L2) | fold slots
    // (fused IQ3; fused IQ2 lays them over the fold warp's state and on)
    int *kmap = reinterpret_cast<int *>(smem_raw);
    uint16_t *gco = reinterpret_cast<uint16_t *>(smem_raw + ((C::KMAP * 4 + 15) & ~15));
    IqWarpSmem<V> *wsm_all = reinterpret_cast<IqWarpSmem<V> *>(reinterpret_cast<uint8_t *>(gco + 256));
    uint8_t *s_lists = reinterpret_cast<uint8_t *>(wsm_all + NW);
    for (int i = threadIdx.x; i < C::KMAP; i += blockDim.x) kmap[i] = g_kmap[i];
    if (V == 0)
        for (int i = threadIdx.x; i < 256; i += blockDim.x) gco[i] = (uint16_t)g_coords[i];
    if (IqSearch<V>::LISTS_SMEM) {
        const uint4 *src4 = static_cast<const uint4 *>(g_lists);
        uint4 *dst4 = reinterpret_cast<uint4 *>(s_lists);
        for (int i = threadIdx.x; i < lists_bytes / 16; i += blockDim.x) dst4[i] = src4[i];
    }
    __syncthreads();
    const void *lists = IqSearch<V>::LISTS_SMEM ? (const void *)s_lists : g_lists;
    const uint16_t *l16 = static_cast<const uint16_t *>(lists);
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    IqWarpSmem<V> &S = wsm_all[wid];
    const int64_t ne0 = a.src.ne0, nsb = ne0 >> 8, total = a.n_rows * nsb;
    constexpr int NWE = NW - 1;
    FuseSmem<NWE> *F = reinterpret_cast<FuseSmem<NWE> *>(
        IqSearch<V>::LISTS_SMEM ? s_lists + ((lists_bytes + 15) & ~15) : reinterpret_cast<uint8_t *>(wsm_all + NWE));
    if constexpr (FUSE) {
        fuse_setup(*F);
        if (wid == NWE) {
            fuse_fold(*F, a, nsb, lane);
            return;
        }
    }
    // sig_in >= 0: the super-block's sigma^2, computed ahead for a batch
    auto unit = [&](int64_t g, float sig_in) {
        const int64_t row = g / nsb;
        const int64_t sbi = g - row * nsb;
        const int64_t col0 = sbi << 8;
        const float *imr = im_row(a.im, ne0, a.row0 + row * a.row_step);
        // ---- P0: load, super-block sigma^2, weights, signs ----
        float v[8];
        load8(a.src, row, col0 + lane * 8, v);
        float sig = sig_in;
        if (sig_in < 0.0f) {
#pragma unroll
            for (int k = 0; k < 8; k++) S.x[lane * 8 + k] = v[k];
            __syncwarp();
            float ssum = 0.0f;
            for (int i = 0; i < 256; i++) ssum += S.x[i] * S.x[i];
            sig = C::SIG2X ? 2.0f * ssum / 256.0f : ssum / 256.0f;
        }
        float base[8];
        load_im8(imr, col0 + lane * 8, base);
        float wv[8];
        // this lane's 8 elements lie in one block: element lane*8+k
        const int eb = (lane * 8) / C::BS, ei = (lane * 8) % C::BS;
#pragma unroll
        for (int k = 0; k < 8; k++) {
            float wt;
            if (V == 2) wt = imr ? base[k] * sqrtf(sig + v[k] * v[k]) : 0.25f * sig + v[k] * v[k];
            else if (V >= 3) wt = imr ? base[k] * sqrtf(sig + v[k] * v[k]) : v[k] * v[k];
            else wt = base[k] * sqrtf(sig + v[k] * v[k]);
            wv[k] = wt;
            S.w[eb * BP + ei + k] = wt;
            S.wa[eb * BP + ei + k] = sqrtf(wt);
        }
        // sign group `lane` = elements lane*8 .. lane*8+7
        {
            float xv8[8];
            int nflip = 0;
            uint32_t sgn = 0;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                if (v[i] >= 0.0f) {
                    xv8[i] = v[i];
                } else {
                    xv8[i] = -v[i];
                    nflip++;
                    sgn |= 1u << i;
                }
            }
            if (C::PARITY && (nflip % 2) != 0) {
                int imin = 0;
                float mn = wv[0] * v[0] * v[0];
#pragma unroll
                for (int i = 1; i < 8; i++) {
                    const float ax = wv[i] * v[i] * v[i];
                    if (ax < mn) { mn = ax; imin = i; }
                }
#pragma unroll
                for (int i = 0; i < 8; i++)
                    if (i == imin) xv8[i] = -xv8[i];
                sgn ^= 1u << imin;
            }
#pragma unroll
            for (int i = 0; i < 8; i++) S.xv[eb * BP + ei + i] = xv8[i];
            S.signs[lane] = (uint8_t)(C::PARITY ? (sgn & 127u) : sgn);
        }
        __syncwarp();
        // ---- P1: per-block max and starting scale ----
        if (C::QP) {  // IQ2_XXS: eight blocks of 32, four lanes each
            const int b = lane >> 2;
            const float s = make_qp_quants32_x4(S.xv + b * BP, S.w + b * BP, S.qpl + b * 32, lane);
            if ((lane & 3) == 0) S.qps[b] = s;
            __syncwarp();
        }
        if (lane < C::NB) {
            const int b = lane;
            const float *xb = S.xv + b * BP;
            float mx = xb[0];
            for (int i = 0; i < C::BS; i++) mx = rmaxf(mx, xb[i]);
            bool live;
            if (V == 0 || V == 1) live = !(mx < kGroupMaxEps);
            else if (V == 2) live = !(mx < kGroupMaxEpsIq2S);
            else if (V == 3) live = !(mx <= kGroupMaxEpsIq3Xxs);
            else live = !(mx <= 0.0f);
            float s0 = 0.0f, ref = mx;
            if (live) {
                if (C::QP) {
                    s0 = S.qps[b];
                    ref = s0 * (float)C::KM;  // eff_max
                    if (ref <= 0.0f) live = false;
                } else {
                    s0 = mx / (float)(2 * C::KM - 1);
                }
            }
            S.live[b] = live ? 1 : 0;
            S.bscale0[b] = s0;
            S.bmax[b] = ref;
        }
        __syncwarp();
        // ---- P2: every (block, trial) job: lattice rounding, neighbour
        // searches, the trial's weighted sums (quant_iq.rs trial loops) ----
        if (COOP) {
            // CJ jobs per chunk, one per lane; the chunk's off-grid groups
            // are searched together
            constexpr int CJ = IqSearch<V>::CJ;
            for (int c0 = 0; c0 < NJ; c0 += CJ) {
                const int j = c0 + lane;
                const int b = j / C::NT, t = j - b * C::NT;
                const bool job = lane < CJ && j < NJ && S.live[b];
                float sc = 0.0f;
                Levels<V> lv;
                int mk[C::NG];
                uint32_t offm = 0;
                if (job) {
                    const float id = ((float)(2 * C::KM - 1) + (float)(C::IS_LO + t) * C::STEP) / S.bmax[b];
                    sc = 1.0f / id;
                    offm = round_block_sel<V>(S, kmap, l16, b * BP, id, sc, (1u << C::NG) - 1, lv, mk, a.status);
                }
                int T;
                const int pos = warp_exclusive_scan(__popc(offm), lane, T);
                if (offm) queue_tasks<V>(S, pos, offm, mk, b * BP, sc);
                __syncwarp();
                if (T > 0) search_tasks<V>(S, T, lists, gco, lane);
                if (job) {
                    take_results<V>(S, pos, offm, lv, a.status);
                    float sx, s2;
                    block_sums<V>(S.xv + b * BP, S.w + b * BP, lv, sx, s2);
                    S.jres[j] = make_float2(sx, s2);
                }
                __syncwarp();
            }
        } else {
            for (int j = lane; j < NJ; j += 32) {
                const int b = j / C::NT, t = j - b * C::NT;
                if (!S.live[b]) continue;
                const float id = ((float)(2 * C::KM - 1) + (float)(C::IS_LO + t) * C::STEP) / S.bmax[b];
                Levels<V> lv;
                int mk[C::NG];
                round_block<V>(S, kmap, l16, b * BP, id, 1.0f / id, (1u << C::NG) - 1, lv, mk, a.status);
                float sx, s2;
                block_sums<V>(S.xv + b * BP, S.w + b * BP, lv, sx, s2);
                S.jres[j] = make_float2(sx, s2);
            }
            __syncwarp();
        }
        // the reference's sequential `sumqx^2 > best*sumq2` chain over the
        // trials, one lane per block
        float cscale = 0.0f;
        int cwin = -1;
        if (lane < C::NB && S.live[lane]) {
            cscale = S.bscale0[lane];
            float cbest = 0.0f;
            for (int tt = 0; tt < C::NT; tt++) {
                const float2 r = S.jres[lane * C::NT + tt];
                if (r.y > 0.0f && r.x * r.x > cbest * r.y) {
                    cscale = r.x / r.y;
                    cbest = cscale * r.x;
                    cwin = tt;
                }
            }
        }
        // the winning trial's lattice points: that trial again, for the
        // blocks that have one
        Levels<V> wl;
        uint32_t woff = 0;
        if constexpr (!COOP) {
            if (lane < C::NB) {
                S.rtodo[lane] = cwin >= 0 ? (1u << C::NG) - 1 : 0u;
                if (cwin >= 0) {
                    const float id = ((float)(2 * C::KM - 1) + (float)(C::IS_LO + cwin) * C::STEP) / S.bmax[lane];
                    S.rid[lane] = id;
                    S.rsc[lane] = 1.0f / id;
                }
            }
            round_groups_lanes<V>(S, kmap, l16, lane, a.status);
            if (cwin >= 0) {
#pragma unroll
                for (int k = 0; k < C::NG; k++) {
                    wl.set_group(k, S.rg[lane * C::NG + k]);
                    woff |= (uint32_t)S.roff[lane * C::NG + k] << k;
                }
            }
        } else {
            float sc = 0.0f;
            int mk[C::NG];
            if (cwin >= 0) {
                const float id = ((float)(2 * C::KM - 1) + (float)(C::IS_LO + cwin) * C::STEP) / S.bmax[lane];
                sc = 1.0f / id;
                woff = round_block_sel<V>(S, kmap, l16, lane * BP, id, sc, (1u << C::NG) - 1, wl, mk, a.status);
            }
            if (COOP) {
                int T;
                const int pos = warp_exclusive_scan(__popc(woff), lane, T);
                if (woff) queue_tasks<V>(S, pos, woff, mk, lane * BP, sc);
                __syncwarp();
                if (T > 0) search_tasks<V>(S, T, lists, gco, lane);
                if (cwin >= 0) take_results<V>(S, pos, woff, wl, a.status);
            }
            __syncwarp();
        }
        // ---- P3: per block: the winner's points, re-projection at the final
        // scale (quant_iq.rs, e.g. 364-384), sign flip and grid indices ----
        {
            const int b = lane;
            const bool blk = lane < C::NB && S.live[b];
            float scale = cscale;
            // on-grid flags start true (IQ3_S: false) and follow the winning trial
            uint32_t off = (V == 4) ? ((1u << C::NG) - 1) : 0u;
            Levels<V> ls;
            if (blk && cwin >= 0) {
                ls = wl;
                off = woff;
            }
            const bool reproject = blk && ((V == 0) ? (scale > 0.0f) : (off != 0 && scale > 0.0f));
            uint32_t offm = 0;
            int mk[C::NG];
            if constexpr (!COOP) {
                const uint32_t todo = (V == 0 || V == 4) ? ((1u << C::NG) - 1) : off;
                if (lane < C::NB) {
                    S.rtodo[b] = reproject ? todo : 0u;
                    S.rid[b] = 1.0f / scale;
                    S.rsc[b] = scale;
                }
                round_groups_lanes<V>(S, kmap, l16, lane, a.status);
                if (reproject) {
#pragma unroll
                    for (int k = 0; k < C::NG; k++)
                        if ((todo >> k) & 1u) ls.set_group(k, S.rg[b * C::NG + k]);
                }
            } else if (reproject) {
                const uint32_t todo = (V == 0 || V == 4) ? ((1u << C::NG) - 1) : off;
                offm = round_block_sel<V>(S, kmap, l16, b * BP, 1.0f / scale, scale, todo, ls, mk, a.status);
            }
            int pos = 0;
            if (COOP) {
                int T;
                pos = warp_exclusive_scan(__popc(offm), lane, T);
                if (offm) queue_tasks<V>(S, pos, offm, mk, b * BP, scale);
                __syncwarp();
                if (T > 0) search_tasks<V>(S, T, lists, gco, lane);
            }
            if (reproject) {
                if (COOP) take_results<V>(S, pos, offm, ls, a.status);
                float sx, s2;
                block_sums<V>(S.xv + b * BP, S.w + b * BP, ls, sx, s2);
                if (s2 > 0.0f) scale = sx / s2;
            }
            if (blk) {
                if (scale < 0.0f) {
                    scale = -scale;
                    for (int k = 0; k < C::NSG; k++) {
                        const uint8_t sg = S.signs[b * C::NSG + k];
                        S.signs[b * C::NSG + k] = C::PARITY ? (uint8_t)((~sg) & 127) : (uint8_t)(~sg);
                    }
                }
#pragma unroll 1
                for (int k = 0; k < C::NG; k++) {
                    const int m = kmap[kmap_index<V>(ls.group(k))];
                    if (m < 0) set_status(a.status, SHC_EOFFGRID);
                    S.gidx[b * C::NG + k] = (uint16_t)(m < 0 ? 0 : m);
                }
                S.bscale[b] = scale;
            } else if (lane < C::NB) {
                for (int k = 0; k < C::NG; k++) S.gidx[b * C::NG + k] = 0;
                for (int k = 0; k < C::NSG; k++) S.signs[b * C::NSG + k] = 0;
                S.bscale[b] = 0.0f;
            }
        }
        __syncwarp();
        // ---- P4: super-block scale and packing, lane b packs block b ----
        {
            uint8_t *o = S.out;
            for (int i = lane; i < C::OUT; i += 32) o[i] = 0;
            // the max of the block scales (NaN-ignoring, -0 < +0: associative,
            // so the butterfly gives the reference's sequential fold)
            float max_scale = lane < C::NB ? S.bscale[lane] : 0.0f;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) max_scale = rmaxf(max_scale, __shfl_xor_sync(0xffffffffu, max_scale, off));
            max_scale = rmaxf(0.0f, max_scale);
            const bool has = max_scale != 0.0f;
            const float d = max_scale / 31.0f;
            const float id = 1.0f / d;
            const int b = lane;
            const bool mine = b < C::NB;
            const int nb_l = mine ? clampi(nearest_int(0.5f * (id * S.bscale[b] - 1.0f)), 0, 15) : 0;
            // block b's scale nibble paired with block b + 1's (even b writes the byte)
            const int nb_pair = nb_l | (__shfl_down_sync(0xffffffffu, nb_l, 1) << 4);
            const bool live = mine && S.live[b];
            __syncwarp();
            auto put16 = [&](int at, uint16_t h) {
                o[at] = (uint8_t)(h & 0xFF);
                o[at + 1] = (uint8_t)(h >> 8);
            };
            auto put32 = [&](int at, uint32_t u) {
                o[at] = (uint8_t)u;
                o[at + 1] = (uint8_t)(u >> 8);
                o[at + 2] = (uint8_t)(u >> 16);
                o[at + 3] = (uint8_t)(u >> 24);
            };
            if (V == 0) {  // IQ2_XXS: the q2 words only reach the output with a nonzero scale
                if (has) {
                    if (lane == 0) put16(0, f16_bits(d));
                    if (mine) {
                        uint32_t q0 = 0, q1 = 0;
                        for (int k = 0; k < 4; k++) {
                            q0 |= (uint32_t)S.gidx[b * 4 + k] << (8 * k);
                            q1 |= (uint32_t)S.signs[b * 4 + k] << (7 * k);
                        }
                        q1 |= (uint32_t)nb_l << 28;
                        put32(2 + 8 * b, q0);
                        put32(6 + 8 * b, q1);
                    }
                }
            } else if (V == 1) {  // IQ2_XS
                if (has) {
                    if (lane == 0) put16(0, f16_bits(d));
                    if (mine) {
                        for (int k = 0; k < 2; k++)
                            put16(2 + 2 * (2 * b + k), (uint16_t)(S.gidx[b * 2 + k] | (S.signs[b * 2 + k] << 9)));
                        if (b % 2 == 0) o[66 + b / 2] = (uint8_t)nb_pair;
                    }
                }
            } else if (V == 2) {  // IQ2_S: grid and sign bytes are written per block
                // high grid bits of blocks b, b + 1 share one byte (two bits per group)
                uint32_t qh = 0;
                if (live) {
                    for (int k = 0; k < 2; k++) {
                        const int i8v = 2 * b + k, gi = S.gidx[b * 2 + k];
                        o[2 + i8v] = (uint8_t)(gi & 255);
                        qh |= (uint32_t)((gi >> 8) << (2 * (i8v % 4)));
                        o[2 + 32 + i8v] = S.signs[b * 2 + k];
                    }
                }
                const uint32_t qh_pair = qh | __shfl_down_sync(0xffffffffu, qh, 1);
                if (mine && b % 2 == 0) o[2 + 64 + b / 2] = (uint8_t)qh_pair;
                if (has) {
                    if (lane == 0) put16(0, f16_bits(d * 0.9875f));
                    if (mine && b % 2 == 0) o[2 + 64 + 8 + b / 2] = (uint8_t)nb_pair;
                }
            } else if (V == 3) {  // IQ3_XXS
                if (live)
                    for (int k = 0; k < 8; k++) o[2 + 8 * b + k] = (uint8_t)S.gidx[b * 8 + k];
                if (has) {
                    if (lane == 0) put16(0, f16_bits(d * 1.0125f));
                    if (mine) {
                        uint32_t sas = 0;
                        if (live)
                            sas = (uint32_t)S.signs[b * 4] | ((uint32_t)S.signs[b * 4 + 1] << 7) |
                                  ((uint32_t)S.signs[b * 4 + 2] << 14) | ((uint32_t)S.signs[b * 4 + 3] << 21);
                        sas |= (uint32_t)nb_l << 28;
                        put32(2 + 64 + 4 * b, sas);
                    }
                }
            } else {  // IQ3_S
                if (live) {
                    uint8_t hi = 0;
                    for (int k = 0; k < 8; k++) {
                        const int gi = S.gidx[b * 8 + k];
                        o[2 + 8 * b + k] = (uint8_t)(gi & 255);
                        hi |= (uint8_t)((gi >> 8) << k);
                    }
                    o[2 + 64 + b] = hi;
                    for (int k = 0; k < 4; k++) o[2 + 64 + 8 + 4 * b + k] = S.signs[b * 4 + k];
                }
                if (has) {
                    if (lane == 0) put16(0, f16_bits(d * 1.033f));
                    if (mine && b % 2 == 0) o[2 + 64 + 8 + 32 + b / 2] = (uint8_t)nb_pair;
                }
            }
        }
        __syncwarp();
        if constexpr (!FUSE)
            store_block(a.dst + row * a.dst_row_bytes + sbi * C::OUT, S.out, C::OUT, a.dst_aligned16 != 0, lane);
        __syncwarp();
    };
    if constexpr (!FUSE) {
        // the warp's super-blocks g0, g0 + st, ... in batches of 32: lane k
        // first folds the sigma^2 of the batch's k-th super-block (the
        // serial sum over its 256 elements, one super-block per lane)
        const int64_t st = (int64_t)gridDim.x * NW;
        for (int64_t g0 = (int64_t)blockIdx.x * NW + wid; g0 < total; g0 += 32 * st) {
            {
                const int64_t gk = g0 + lane * st;
                float ssum = 0.0f;
                if (gk < total) {
                    const int64_t row = gk / nsb, col0 = (gk - row * nsb) << 8;
#pragma unroll 4
                    for (int m = 0; m < 32; m++) {
                        float v[8];
                        load8(a.src, row, col0 + m * 8, v);
#pragma unroll
                        for (int k = 0; k < 8; k++) ssum += v[k] * v[k];
                    }
                }
                S.sigb[lane] = C::SIG2X ? 2.0f * ssum / 256.0f : ssum / 256.0f;
            }
            __syncwarp();
            for (int k = 0; k < 32 && g0 + k * st < total; k++) unit(g0 + k * st, S.sigb[k]);
        }
    } else {
        constexpr uint32_t TYPE = V == 0 ? SHC_TYPE_IQ2_XXS : V == 1 ? SHC_TYPE_IQ2_XS : V == 2 ? SHC_TYPE_IQ2_S
                                  : V == 3 ? SHC_TYPE_IQ3_XXS : SHC_TYPE_IQ3_S;
        FuseIter<NWE> it(a, nsb, wid);
        uint32_t fk = 0;
        while (it.next()) {
            if (it.valid) unit(it.row * nsb + it.unit, -1.0f);
            fuse_emit<TYPE, 0>(*F, wid, fk, it.valid, a, it.row, it.unit, S.out, lane);
        }
    }
}

template <int V, bool FUSE>
static cudaError_t launch_lattice(EncArgs a, const IqTables &iq, int num_sms, cudaStream_t st) {
    using C = IqCfg<V>;
    constexpr int NW = IqWarps<V, FUSE>::value;
    const size_t ws_end = ((C::KMAP * 4 + 15) & ~(size_t)15) + 512 + NW * sizeof(IqWarpSmem<V>);
    size_t smem = ws_end + (IqSearch<V>::LISTS_SMEM ? (((size_t)iq.lists_bytes[V] + 15) & ~(size_t)15) : 0);
    if (FUSE) {
        if (IqSearch<V>::LISTS_SMEM) smem += sizeof(FuseSmem<NW - 1>);
        else smem = std::max(smem, ws_end - sizeof(IqWarpSmem<V>) + sizeof(FuseSmem<NW - 1>));
    }
    auto fn = enc_iq_lattice_kernel<V, FUSE>;
    int per_sm = 1;
    cudaError_t e = resident_blocks((const void *)fn, NW * 32, smem, &per_sm);
    if (e != cudaSuccess) return e;
    const int64_t upr = a.src.ne0 / 256;
    const int64_t cap = (int64_t)num_sms * per_sm;
    int64_t grid;
    if (FUSE) {
        a.fuse_rows = fuse_rows_per_group(a.n_rows, upr, NW - 1, cap);
        grid = (a.n_rows + a.fuse_rows - 1) / a.fuse_rows;
    } else {
        grid = (a.n_rows * upr + NW - 1) / NW;
    }
    if (grid > cap) grid = cap;
    if (grid < 1) grid = 1;
    fn<<<(unsigned)grid, NW * 32, smem, st>>>(a, iq.dkmap[V], iq.lists[V], iq.lists_bytes[V], iq.grid_coords[V]);
    return cudaGetLastError();
}

template <bool XS, bool FUSE>
static cudaError_t launch_iq4(EncArgs a, int num_sms, cudaStream_t st) {
    auto fn = enc_iq4_kernel<XS, FUSE>;
    const size_t smem = FUSE ? sizeof(FuseSmem<7>) : 0;
    int per_sm = 1;
    cudaError_t e = resident_blocks((const void *)fn, 256, smem, &per_sm);
    if (e != cudaSuccess) return e;
    const int64_t cap = (int64_t)num_sms * per_sm;
    int64_t grid;
    if (FUSE) {
        a.fuse_rows = fuse_rows_per_group(a.n_rows, (a.src.ne0 + 255) / 256, 7, cap);
        grid = (a.n_rows + a.fuse_rows - 1) / a.fuse_rows;
    } else {
        const int64_t units = XS ? a.n_rows * (a.src.ne0 / 256) : (a.n_rows * (a.src.ne0 / 32) + 7) / 8;
        grid = (units + 7) / 8;
    }
    if (grid > cap) grid = cap;
    if (grid < 1) grid = 1;
    fn<<<(unsigned)grid, 256, smem, st>>>(a);
    return cudaGetLastError();
}

bool iq_supported(uint32_t type) {
    switch (type) {
    case SHC_TYPE_IQ4_NL: case SHC_TYPE_IQ4_XS: case SHC_TYPE_IQ2_XXS: case SHC_TYPE_IQ2_XS: case SHC_TYPE_IQ2_S:
    case SHC_TYPE_IQ3_XXS: case SHC_TYPE_IQ3_S:
        return true;
    default:
        return false;
    }
}

cudaError_t launch_iq(uint32_t type, const EncArgs &a, const IqTables &iq, int num_sms, cudaStream_t st) {
    switch (type) {
    case SHC_TYPE_IQ4_NL: return launch_iq4<false, false>(a, num_sms, st);
    case SHC_TYPE_IQ4_XS: return launch_iq4<true, false>(a, num_sms, st);
    case SHC_TYPE_IQ2_XXS: return launch_lattice<0, false>(a, iq, num_sms, st);
    case SHC_TYPE_IQ2_XS: return launch_lattice<1, false>(a, iq, num_sms, st);
    case SHC_TYPE_IQ2_S: return launch_lattice<2, false>(a, iq, num_sms, st);
    case SHC_TYPE_IQ3_XXS: return launch_lattice<3, false>(a, iq, num_sms, st);
    case SHC_TYPE_IQ3_S: return launch_lattice<4, false>(a, iq, num_sms, st);
    default: return cudaErrorNotSupported;
    }
}

cudaError_t launch_iq_fused(uint32_t type, const EncArgs &a, const IqTables &iq, int num_sms, cudaStream_t st) {
    if (!a.err || a.n_rows < 1) return cudaErrorInvalidValue;
    switch (type) {
    case SHC_TYPE_IQ4_NL: return launch_iq4<false, true>(a, num_sms, st);
    case SHC_TYPE_IQ4_XS: return launch_iq4<true, true>(a, num_sms, st);
    case SHC_TYPE_IQ2_XXS: return launch_lattice<0, true>(a, iq, num_sms, st);
    case SHC_TYPE_IQ2_XS: return launch_lattice<1, true>(a, iq, num_sms, st);
    case SHC_TYPE_IQ2_S: return launch_lattice<2, true>(a, iq, num_sms, st);
    case SHC_TYPE_IQ3_XXS: return launch_lattice<3, true>(a, iq, num_sms, st);
    case SHC_TYPE_IQ3_S: return launch_lattice<4, true>(a, iq, num_sms, st);
    default: return cudaErrorNotSupported;
    }
}

}  // namespace shc
