// Fused error table: the epilogue that turns an encoder's codes, still in
// shared memory, into the weighted squared error of row_error
// (quant.rs:618-630): err = sum_i f64(w_i) * d_i * d_i, d_i = f64(x_i - x^_i),
// folded in element order.  The codes never leave the SM.
//
// A fused launch cuts its rows into groups of R consecutive rows; a CTA owns
// whole groups.  A group's units (256-element chunks of a row) are dealt
// column-major, item i = unit i / R' of row i % R' (R' = the group's row
// count), so the group's rows advance together.  Stage j gives item
// j * NWE + w to encoder warp w; the CTA's last warp folds.  Encoder warp w
// writes its item's terms f64(w_i) * d_i * d_i (exact per element, 32 lanes
// at once) into its slot and arrives on full[w]; the fold warp waits for the
// stage's slots, lane r adds up the slots of row r in item order (so each row
// is one serial f64 chain in column order, as the reference folds it), then
// arrives on empty[w].  A
// slot is rewritten only after its previous contents were folded, which the
// encoder waits for after encoding its next item: the fold of stage j runs
// while stage j + 1 encodes.
//
// Every wait is bounded: after kFuseWaitNs, or once another warp gave up, a
// wait sets SHC_ETIMEOUT in the status word and returns, and every later
// wait of the CTA returns at once, so the kernel always finishes.
#pragma once
#include "decode.cuh"
#include "kernels.cuh"

namespace shc {

constexpr int kFuseStride = 258;  // doubles per slot: 256 + 2, so slots start on different banks
constexpr unsigned long long kFuseWaitNs = 2000000000ull;

template <int NWE>
struct __align__(16) FuseSmem {
    double t[NWE][kFuseStride];
    unsigned long long full[NWE];   // encoder warp w -> fold warp, 32 arrivals per phase
    unsigned long long empty[NWE];  // fold warp -> encoder warp w, 32 arrivals per phase
    int abort;
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(unsigned long long *b, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(unsigned long long *b) {
    asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.shared::cta.b64 st, [%0];\n}" ::"r"(smem_u32(b)) : "memory");
}
// One bounded try: the thread sleeps in hardware until the phase completes or
// about kFuseSuspendNs pass (so a waiting warp takes no issue slots).
constexpr uint32_t kFuseSuspendNs = 1000000;
__device__ __forceinline__ bool mbar_test(unsigned long long *b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity), "r"(kFuseSuspendNs)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Wait for the phase of parity `parity` of barrier b to complete (bounded).
static __device__ __noinline__ void mbar_wait(unsigned long long *b, uint32_t parity, volatile int *abort, int *status) {
    if (mbar_test(b, parity)) return;
    const unsigned long long t0 = global_ns();
    while (!mbar_test(b, parity)) {
        if (*abort) return;
        if (global_ns() - t0 > kFuseWaitNs) {
            *abort = 1;
            set_status(status, SHC_ETIMEOUT);
            return;
        }
    }
}

// Barriers initialised by thread 0, visible to every warp after the
// __syncthreads() that ends this call (every thread of the CTA calls it).
template <int NWE>
__device__ __forceinline__ void fuse_setup(FuseSmem<NWE> &F) {
    if (threadIdx.x == 0) {
        for (int w = 0; w < NWE; w++) {
            mbar_init(&F.full[w], 32);
            mbar_init(&F.empty[w], 32);
        }
        F.abort = 0;
    }
    __syncthreads();
}

// The groups of a fused launch: rows [grp * R, min(grp * R + R, n_rows)),
// upr units per row.
struct FuseGroups {
    int64_t n_rows, upr, R, ngrp;
    __device__ FuseGroups(const EncArgs &a, int64_t units_per_row)
        : n_rows(a.n_rows), upr(units_per_row), R(a.fuse_rows), ngrp((a.n_rows + a.fuse_rows - 1) / a.fuse_rows) {}
    __device__ void group(int64_t grp, int64_t &r0, int64_t &reff, int64_t &items) const {
        r0 = grp * R;
        reff = n_rows - r0 < R ? n_rows - r0 : R;
        items = reff * upr;
    }
};

// Encoder warp w's items, stage by stage (every encoder warp of the CTA
// takes the same number of stages; past a group's last item `valid` is
// false).
template <int NWE>
struct FuseIter {
    FuseGroups G;
    int w;
    int64_t grp, r0 = 0, reff = 1, items = 0, j = 0, nst = 0;
    bool valid = false;
    int64_t row = 0, unit = 0;
    __device__ FuseIter(const EncArgs &a, int64_t upr, int warp)
        : G(a, upr), w(warp), grp((int64_t)blockIdx.x - (int64_t)gridDim.x) {}
    __device__ bool next() {
        while (j >= nst) {
            grp += gridDim.x;
            if (grp >= G.ngrp) return false;
            G.group(grp, r0, reff, items);
            nst = (items + NWE - 1) / NWE;
            j = 0;
        }
        const int64_t idx = j * NWE + w;
        j++;
        valid = idx < items;
        row = valid ? r0 + idx % reff : r0;
        unit = valid ? idx / reff : 0;
        return true;
    }
};

// Encoder side: the terms f64(w) * d * d, d = x - decode(codes), of this
// warp's item into its slot (w = the imatrix weight, 1 without one).  TYPE is the encoded ggml type; BB the bytes of one 32-element
// block for the 32-element block types (a unit is then up to eight blocks
// back to back in `codes`), 0 when `codes` holds one 256-element block.
// Lane l takes elements 32 (l / 4) + 8 (l % 4) + [0, 8).
template <uint32_t TYPE, int BB, int NWE>
__device__ __forceinline__ void fuse_emit(FuseSmem<NWE> &F, int w, uint32_t &k, bool valid, const EncArgs &a,
                                          int64_t row, int64_t unit, const uint8_t *codes, int lane) {
    if (k >= 1) mbar_wait(&F.empty[w], (k - 1) & 1u, &F.abort, a.status);
    if (valid) {
        const int sub = lane >> 2, qq = lane & 3;
        const int64_t c0 = unit * 256;
        const int e0 = sub * 32 + qq * 8;
        if (c0 + e0 < a.src.ne0) {
            float y[32];
            if (BB) decode_sub32(TYPE, codes + sub * BB, 0, y);
            else decode_sub32(TYPE, codes, sub, y);
            float xv[8], wv[8];
            load8(a.src, row, c0 + e0, xv);
            const float *imr = im_row(a.im, a.src.ne0, a.row0 + row * a.row_step);
            load_im8(imr, c0 + e0, wv);
            double tv[8];
#pragma unroll
            for (int t = 0; t < 8; t++) {
                const float yv = qq == 0 ? y[t] : qq == 1 ? y[8 + t] : qq == 2 ? y[16 + t] : y[24 + t];
                const double dd = (double)(xv[t] - yv);
                const double wd = imr ? (double)wv[t] : 1.0;
                tv[t] = wd * dd * dd;
            }
            double2 *dst = reinterpret_cast<double2 *>(&F.t[w][e0]);
#pragma unroll
            for (int t = 0; t < 4; t++) dst[t] = make_double2(tv[2 * t], tv[2 * t + 1]);
        }
    }
    __syncwarp();
    mbar_arrive(&F.full[w]);
    k++;
}

// Encoder side for the elementwise types (F32, F16, BF16): the "codes" are
// the row itself, round-tripped through TYPE (quant.rs:546-560).
template <uint32_t TYPE, int NWE>
__device__ __forceinline__ void fuse_emit_plain(FuseSmem<NWE> &F, int w, uint32_t &k, bool valid, const EncArgs &a,
                                                int64_t row, int64_t unit, int lane) {
    if (k >= 1) mbar_wait(&F.empty[w], (k - 1) & 1u, &F.abort, a.status);
    if (valid) {
        const int64_t c0 = unit * 256;
        const int e0 = lane * 8;
        if (c0 + e0 < a.src.ne0) {
            float xv[8], wv[8];
            load8(a.src, row, c0 + e0, xv);
            const float *imr = im_row(a.im, a.src.ne0, a.row0 + row * a.row_step);
            load_im8(imr, c0 + e0, wv);
            double tv[8];
#pragma unroll
            for (int t = 0; t < 8; t++) {
                const double dd = (double)(xv[t] - roundtrip_plain(TYPE, xv[t]));
                const double wd = imr ? (double)wv[t] : 1.0;
                tv[t] = wd * dd * dd;
            }
            double2 *dst = reinterpret_cast<double2 *>(&F.t[w][e0]);
#pragma unroll
            for (int t = 0; t < 4; t++) dst[t] = make_double2(tv[2 * t], tv[2 * t + 1]);
        }
    }
    __syncwarp();
    mbar_arrive(&F.full[w]);
    k++;
}

// Fold warp: per row of each group, sum f64(w) * d * d over the row's
// elements in order, one lane per row; err[row] for every row of the view.
template <int NWE>
__device__ void fuse_fold(FuseSmem<NWE> &F, const EncArgs &a, int64_t upr, int lane) {
    const FuseGroups G(a, upr);
    const int64_t ne0 = a.src.ne0;
    int64_t K = 0;  // stages of this CTA
    for (int64_t grp = blockIdx.x; grp < G.ngrp; grp += gridDim.x) {
        int64_t r0, reff, items;
        G.group(grp, r0, reff, items);
        K += (items + NWE - 1) / NWE;
    }
    int64_t k = 0;
    for (int64_t grp = blockIdx.x; grp < G.ngrp; grp += gridDim.x) {
        int64_t r0, reff, items;
        G.group(grp, r0, reff, items);
        const int64_t nst = (items + NWE - 1) / NWE;
        const bool mine = lane < reff;
        double s = 0.0;
        for (int64_t j = 0; j < nst; j++, k++) {
            for (int w = 0; w < NWE; w++) mbar_wait(&F.full[w], (uint32_t)(k & 1), &F.abort, a.status);
            if (mine) {
                const int64_t m = (j * NWE) % reff;
                for (int64_t w = (lane - m + reff) % reff; w < NWE; w += reff) {
                    const int64_t idx = j * NWE + w;
                    if (idx >= items) break;
                    const int64_t c0 = (idx / reff) * 256;
                    const int n = (int)(ne0 - c0 < 256 ? ne0 - c0 : 256);
                    const double2 *tp = reinterpret_cast<const double2 *>(F.t[w]);
#pragma unroll 4
                    for (int e = 0; e < n / 2; e += 4) {
                        const double2 t0 = tp[e], t1 = tp[e + 1], t2 = tp[e + 2], t3 = tp[e + 3];
                        s += t0.x;
                        s += t0.y;
                        s += t1.x;
                        s += t1.y;
                        s += t2.x;
                        s += t2.y;
                        s += t3.x;
                        s += t3.y;
                    }
                }
            }
            __syncwarp();
            if (k + 1 < K)
                for (int w = 0; w < NWE; w++) mbar_arrive(&F.empty[w]);
        }
        // a NaN error is stored as the default quiet NaN (payloads are not
        // part of the result)
        if (mine) a.err[r0 + lane] = s == s ? s : __longlong_as_double(0x7FF8000000000000ll);
    }
}

// Rows per group for a fused launch over n_rows rows of upr units with NWE
// encoder warps per CTA and `ctas` resident CTAs: small groups keep every
// resident CTA busy, groups of at least NWE items keep every encoder warp
// busy, and a group has at most 32 rows (one fold lane each).
inline int64_t fuse_rows_per_group(int64_t n_rows, int64_t upr, int nwe, int64_t ctas) {
    int64_t r = (n_rows + ctas - 1) / (ctas > 0 ? ctas : 1);
    const int64_t fill = (nwe + upr - 1) / upr;
    if (r < fill) r = fill;
    if (r > 32) r = 32;
    if (r > n_rows) r = n_rows;
    return r < 1 ? 1 : r;
}

}  // namespace shc
