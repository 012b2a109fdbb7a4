// Device-side scalar semantics shared by every encoder kernel.
//
// The encoders must reproduce the reference's Rust f32 arithmetic bit for bit
// (src/quant.rs, src/quant_iq.rs).  The library is compiled with
// -fmad=false -prec-div=true -prec-sqrt=true -ftz=false, so every a*b+c below
// is a separately rounded multiply and add, `/` and sqrtf are IEEE-correct and
// subnormals are kept.  The helpers here pin the remaining Rust semantics:
//   nearest_int  f32::round (half away from zero) then a saturating `as i32`
//   rmaxf/rminf  f32::max / f32::min: NaN-ignoring, with -0 < +0 (the aarch64
//                FMAXNM/FMINNM result)
//   f16 bits     half::f16::from_f32, IEEE round-to-nearest-even
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "shoehorn_cuda.h"

namespace shc {

constexpr float kGroupMaxEps = 1e-15f;
constexpr float kGroupMaxEpsIq3Xxs = 1e-8f;
constexpr float kGroupMaxEpsIq2S = 1e-8f;

// quant.rs:16 nearest_int: `x.round() as i32` (saturating, NaN -> 0).
__device__ __forceinline__ int nearest_int(float x) {
    float r = roundf(x);
    if (r != r) return 0;
    if (r >= 2147483648.0f) return 2147483647;
    if (r <= -2147483648.0f) return (-2147483647 - 1);
    return (int)r;
}

// Rounding without the conversion pipe.  roundf/floorf/rintf and float<->int
// conversions issue at a quarter of the FP32 add rate per SM sub-partition on
// sm_100; the helpers below round with three full-rate adds.  They rest on two
// exact identities of IEEE binary32 arithmetic:
//   (a) for 0 <= z < 2^23, RD(z + 2^23) = 2^23 + floor(z) (the floats of
//       [2^23, 2^24) are the integers) and subtracting 2^23 again is exact;
//   (b) for t >= 0, floor(RZ(t + 1/2)) = floor(t + 1/2): the exact sum s is
//       >= 1/2, RZ never crosses the integer below s, and stays below s.
// Hence floor_half_up(t) = floor(t + 1/2) = round-half-away-from-zero(t) for
// 0 <= t < 2^23 - 1/2.  For t >= 2^23 - 1/2 the result is >= 2^23 - 1 (callers
// clamp to bounds far below that); for t < 0 it is <= 0 (callers clamp at 0
// or use the magnitude); NaN and +-inf pass through.
__device__ __forceinline__ float floor_half_up(float t) {
    return __fadd_rn(__fadd_rd(__fadd_rz(t, 0.5f), 8388608.0f), -8388608.0f);
}
__device__ __forceinline__ float2 floor_half_up2(float2 t) {
    return __fadd2_rn(__fadd2_rd(__fadd2_rz(t, make_float2(0.5f, 0.5f)), make_float2(8388608.0f, 8388608.0f)),
                      make_float2(-8388608.0f, -8388608.0f));
}
// Packed f32x2 arithmetic (two IEEE-rounded f32 operations per instruction).
// Code generation for sm_100 contracts a packed multiply that feeds a packed
// round-to-nearest add into a fused multiply-add in some operand patterns,
// even under -fmad=false, which changes the rounding of the sum.  The
// encoders therefore use packed multiplies only where their results feed
// multiplies or scalar adds, and packed round-to-nearest adds only on
// operands that are not products; scalar multiply/add pairs and
// directed-rounding adds are not contracted.  The byte-parity tests over
// thousands of super-blocks guard this rule.

// f32::round for |x| < 2^23 - 1/2 (half away from zero, sign of x kept, so
// -0.3 -> -0); larger magnitudes come out >= 2^23 - 1 with the sign of x.
__device__ __forceinline__ float round_away_small(float x) { return copysignf(floor_half_up(fabsf(x)), x); }

// nearest_int(x).clamp(0, hi) kept in float, for integer hi < 2^22.  Every x
// is covered: x >= 0 rounds half away (floor_half_up), x in [-1/2, 0) gives 0
// like the clamped -0/-1 of f32::round, x < -1/2 gives <= 0 -> 0, NaN -> 0
// (fmaxf returns the non-NaN operand, as the saturating cast maps NaN to 0),
// +inf -> hi.  A zero result is +0 (the last add of floor_half_up rounds
// 2^23 - 2^23 to +0).
__device__ __forceinline__ float round_clamp0_f(float x, float hi) {
    return fminf(fmaxf(floor_half_up(x), 0.0f), hi);
}
// nearest_int(x).clamp(0, hi) as an integer, for integer 0 < hi < 256,
// without a conversion instruction: RD(RZ(x + 1/2) + 2^23) is 2^23 + the
// rounded value (identities (a), (b) above), clamped in that biased form to
// [2^23, 2^23 + hi] (NaN and everything below 2^23 go to the lower bound),
// whose low mantissa bits are the result.
__device__ __forceinline__ int round_clamp0_i(float x, float hi) {
    const float b = __fadd_rd(__fadd_rz(x, 0.5f), 8388608.0f);
    return (int)(__float_as_uint(fminf(fmaxf(b, 8388608.0f), 8388608.0f + hi)) & 0xFFu);
}
// (2l+1) as a float for a small non-negative integer l, without a conversion
// instruction: the integer in the low mantissa bits of 2^23, minus 2^23.
__device__ __forceinline__ float odd_level(uint32_t l) {
    return __uint_as_float(0x4B000001u | (l << 1)) - 8388608.0f;
}

// nearest_int(x).clamp(lo, hi) in float for lo < 0 < hi, |lo|, hi < 2^22:
// NaN must map to 0 (not lo) as the saturating cast does.
__device__ __forceinline__ float round_clamp_f(float x, float lo, float hi) {
    float r = round_away_small(x);
    r = (r != r) ? 0.0f : r;
    return fminf(fmaxf(r, lo), hi);
}

__device__ __forceinline__ int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

__device__ __forceinline__ float rmaxf(float a, float b) {
    if (a != a) return b;
    if (b != b) return a;
    if (a > b) return a;
    if (b > a) return b;
    return signbit(a) ? b : a;
}
__device__ __forceinline__ float rminf(float a, float b) {
    if (a != a) return b;
    if (b != b) return a;
    if (a < b) return a;
    if (b < a) return b;
    return signbit(a) ? a : b;
}

__device__ __forceinline__ uint16_t f16_bits(float x) { return __half_as_ushort(__float2half_rn(x)); }
__device__ __forceinline__ float f16_val(uint16_t h) { return __half2float(__ushort_as_half(h)); }

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) { return __uint_as_float(((uint32_t)b) << 16); }

// Device status word: first nonzero code wins (atomicCAS from 0).
__device__ __forceinline__ void set_status(int *status, int code) {
    if (status) atomicCAS(status, 0, code);
}

// Row source: the reference feeds encoders f32 rows decoded from the model's
// storage type (main.rs:397-406 via quant.rs:581 decode_row).
struct RowSrc {
    const void *ptr;
    int src_type;  // SHC_SRC_F32 / SHC_SRC_F16 / SHC_SRC_BF16
    int64_t ne0;
    int64_t row_stride;  // elements between consecutive rows
};

// Load 8 consecutive source elements starting at (row, col) as f32.
// col is a multiple of 8; the row base is 16-byte aligned for BF16/F16 and
// 32-byte aligned for F32 (checked on the host before launch).
__device__ __forceinline__ void load8(const RowSrc &s, int64_t row, int64_t col, float v[8]) {
    if (s.src_type == SHC_SRC_BF16) {
        const uint4 q = __ldg(reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(s.ptr) + row * s.row_stride + col));
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int k = 0; k < 4; k++) {
            v[2 * k] = __uint_as_float(w[k] << 16);
            v[2 * k + 1] = __uint_as_float(w[k] & 0xFFFF0000u);
        }
    } else if (s.src_type == SHC_SRC_F16) {
        const uint4 q = __ldg(reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(s.ptr) + row * s.row_stride + col));
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int k = 0; k < 4; k++) {
            v[2 * k] = f16_val((uint16_t)(w[k] & 0xFFFF));
            v[2 * k + 1] = f16_val((uint16_t)(w[k] >> 16));
        }
    } else {
        const float4 *p = reinterpret_cast<const float4 *>(static_cast<const float *>(s.ptr) + row * s.row_stride + col);
        const float4 a = __ldg(p), b = __ldg(p + 1);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    }
}

__device__ __forceinline__ float load1(const RowSrc &s, int64_t row, int64_t col) {
    if (s.src_type == SHC_SRC_BF16) return bf16_bits_to_f32(static_cast<const uint16_t *>(s.ptr)[row * s.row_stride + col]);
    if (s.src_type == SHC_SRC_F16) return f16_val(static_cast<const uint16_t *>(s.ptr)[row * s.row_stride + col]);
    return static_cast<const float *>(s.ptr)[row * s.row_stride + col];
}

// imatrix.rs:124-141 row_slice, as a column-weight pointer for a global row
// index (nullptr means "no imatrix": the per-type fallback weights apply).
struct ImSrc {
    const float *ptr;
    int64_t len;
    int64_t rows_per_mat;
};
__device__ __forceinline__ const float *im_row(const ImSrc &im, int64_t ne0, int64_t grow) {
    if (!im.ptr) return nullptr;
    if (im.len == ne0) return im.ptr;
    if (im.rows_per_mat > 0 && im.len % ne0 == 0) {
        int64_t mat = grow / im.rows_per_mat;
        int64_t n_mats = im.len / ne0;
        int64_t m = mat < n_mats - 1 ? mat : n_mats - 1;
        return im.ptr + (m > 0 ? m : 0) * ne0;
    }
    return nullptr;
}

// Eight imatrix weights at col (1.0 without an imatrix); 32-byte aligned.
__device__ __forceinline__ void load_im8(const float *imr, int64_t col, float b[8]) {
    if (imr) {
        const float4 *p = reinterpret_cast<const float4 *>(imr + col);
        const float4 a0 = __ldg(p), a1 = __ldg(p + 1);
        b[0] = a0.x; b[1] = a0.y; b[2] = a0.z; b[3] = a0.w;
        b[4] = a1.x; b[5] = a1.y; b[6] = a1.z; b[7] = a1.w;
    } else {
#pragma unroll
        for (int k = 0; k < 8; k++) b[k] = 1.0f;
    }
}

// Store nbytes of a shared-memory staged block to global memory, 16 B per
// lane when both ends are 16-byte aligned, else 2 B or 1 B per lane.
__device__ __forceinline__ void store_block(uint8_t *dstp, const uint8_t *sp, int nbytes, bool aligned16, int lane) {
    if (aligned16 && (nbytes & 15) == 0 && ((uintptr_t)dstp & 15) == 0) {
        for (int i = lane; i < nbytes / 16; i += 32)
            reinterpret_cast<uint4 *>(dstp)[i] = reinterpret_cast<const uint4 *>(sp)[i];
    } else if ((nbytes & 1) == 0 && ((uintptr_t)dstp & 1) == 0) {
        for (int i = lane; i < nbytes / 2; i += 32)
            reinterpret_cast<uint16_t *>(dstp)[i] = reinterpret_cast<const uint16_t *>(sp)[i];
    } else {
        for (int i = lane; i < nbytes; i += 32) dstp[i] = sp[i];
    }
}

}  // namespace shc
