// K-quant and Q8_0 encoders for sm_100a.
//
// Parity contract: every kernel reproduces src/quant.rs bit for bit.  The
// scale searches evaluate candidate grids in parallel (one lane owns one
// (sub-block, candidate) pair and folds its sums serially over the elements,
// in the reference's order) and then reproduce the reference's sequential
// selection: a strict `err < best_err` chain is an argmin with first-index
// tie-break (warp shuffles, or a shared-memory atomicMin on (error, grid));
// the cross-multiplied `sumlx^2 > best*suml2` chain of make_qx_quants is
// replayed serially.  The make_qkx3_quants kernels skip grids whose level
// vector repeats the previous grid's, which cannot change either choice.
//
// Work decomposition: one warp per 256-element super-block (grid-stride over
// all super-blocks of the tensor), 128-bit loads of the source row into
// registers/shared memory, the imatrix slice read through the read-only path.
#include <map>
#include <mutex>
#include <tuple>

#include "fuse.cuh"
#include "kernels.cuh"

namespace shc {

// ---------------------------------------------------------------------------
// Row sigma^2 (quant.rs:153-155): sequential f32 fold of x^2 over the whole
// row, then / ne0.  The fold is order-dependent, so one thread owns one row
// and its adds form one dependent chain (4 cycles each: 29 us for a 14336
// row, measured 4.1 cycles per dependent add).  A block owns 32 rows and has
// kSigLoaders + 1 warps: the loaders stream tiles of 32 rows x 512 bytes into
// a kSigStages-deep shared-memory ring with cp.async (16-byte chunks, one
// row's 512 B per instruction, coalesced; the three loaders copy 11, 11 and
// 10 of the tile's 32 rows, keeping that many times the copies in flight
// that one warp would); the folder (warp 0, lane r = row r) only reads its
// row from the ring, unpacks, squares (packed) and adds.  It reads the next
// group of eight chunks into registers before adding the current group, so
// the shared-memory latency (long while the loaders' copies land) stays off
// the add chain.  The warps hand stages over through named barriers counting
// all of them: FULL(s) after the loaders' copies into stage s landed, EMPTY(s)
// after the folder read it.  The folder waits for the next tile's FULL before
// it releases the current tile's EMPTY, so the loaders announce their oldest
// landed tile before they wait for a free stage; every warp walks the same
// tiles, so every barrier is met (the call order is replayed on the CPU by
// tests/test_sigma_protocol.py).  Chunk (row r, j) sits in slot j*32 + r so
// that lane r reads its row 16 bytes at a time without bank conflicts.
// Measured on the 4096 x 14336 sweep tensor: 86 us with one loader and
// 128-byte tiles, 78 us with four loaders, 60 us with the register-prefetched
// groups, 57.6 us (launch-list mean) with the folder alone on its
// sub-partition, against the 30 us chain.
// ---------------------------------------------------------------------------
constexpr int kSigStages = 6;
constexpr int kSigLoaders = 3;
constexpr int kSigThreads = 32 * (kSigLoaders + 1);
constexpr int kSigChunks = 32;  // 16-byte chunks of each row per tile
constexpr size_t kSigSmem = (size_t)kSigStages * kSigChunks * 32 * 16;  // 96 KB

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }
// Named barrier `id` over all the block's warps.
__device__ __forceinline__ void bar_sync_all(int id) {
    asm volatile("bar.sync %0, %1;\n" ::"r"(id), "n"(kSigThreads) : "memory");
}
__device__ __forceinline__ void bar_arrive_all(int id) {
    asm volatile("bar.arrive %0, %1;\n" ::"r"(id), "n"(kSigThreads) : "memory");
}
__device__ __forceinline__ int sig_full(int s) { return 1 + s; }
__device__ __forceinline__ int sig_empty(int s) { return 1 + kSigStages + s; }

// Squares of the 8 elements in one 16-byte chunk (4 for F32), folded into s
// in element order; the products are packed, the adds stay serial.
template <int SRC>
__device__ __forceinline__ void sigma_fold(const uint4 q, float &s) {
    const uint32_t wv[4] = {q.x, q.y, q.z, q.w};
    if (SRC == SHC_SRC_F32) {
        const float2 p0 = __fmul2_rn(make_float2(__uint_as_float(wv[0]), __uint_as_float(wv[1])),
                                     make_float2(__uint_as_float(wv[0]), __uint_as_float(wv[1])));
        const float2 p1 = __fmul2_rn(make_float2(__uint_as_float(wv[2]), __uint_as_float(wv[3])),
                                     make_float2(__uint_as_float(wv[2]), __uint_as_float(wv[3])));
        s = __fadd_rn(s, p0.x);
        s = __fadd_rn(s, p0.y);
        s = __fadd_rn(s, p1.x);
        s = __fadd_rn(s, p1.y);
    } else {
#pragma unroll
        for (int k = 0; k < 4; k++) {
            float2 v;
            if (SRC == SHC_SRC_BF16) v = make_float2(__uint_as_float(wv[k] << 16), __uint_as_float(wv[k] & 0xFFFF0000u));
            else v = make_float2(f16_val((uint16_t)(wv[k] & 0xFFFF)), f16_val((uint16_t)(wv[k] >> 16)));
            const float2 p = __fmul2_rn(v, v);
            s = __fadd_rn(s, p.x);
            s = __fadd_rn(s, p.y);
        }
    }
}

template <int SRC>
__global__ void __launch_bounds__(kSigThreads) row_sigma2_kernel(RowSrc src, int64_t n_rows, float *out) {
    extern __shared__ __align__(16) uint4 sig_ring[];  // [kSigStages][kSigChunks * 32]
    auto ring = [&](int64_t t) { return sig_ring + (t % kSigStages) * (kSigChunks * 32); };
    const int lane = threadIdx.x & 31;
    // warp 0 folds, alone on its scheduler sub-partition (warps are spread
    // over the four by warp index; a loader beside it cost 4 us), warps 1..
    // kSigLoaders load
    const int lw = (int)(threadIdx.x >> 5) - 1;
    const bool loader = lw >= 0;
    const int64_t rbase = (int64_t)blockIdx.x * 32;
    const int64_t ne0 = src.ne0;
    constexpr int esz = SRC == SHC_SRC_F32 ? 4 : 2;
    constexpr int per_chunk = 16 / esz;            // elements per 16-byte chunk
    constexpr int64_t tile_cols = kSigChunks * per_chunk;  // 512 bytes of every row per tile
    const int64_t ntiles = (ne0 + tile_cols - 1) / tile_cols;
    const int64_t full_tiles = ne0 / tile_cols;
    if (loader) {
        const char *base = static_cast<const char *>(src.ptr);
        const int64_t row_bytes = src.row_stride * esz;
        // this lane's chunks of a tile: 16-byte column `lane` of rows lw, lw + kSigLoaders, ...
        const int j = lane;
        auto issue = [&](int64_t t) {
            uint4 *slot = ring(t);
            const int64_t col = t * tile_cols + (int64_t)j * per_chunk;
            if (col < ne0) {
#pragma unroll
                for (int i = 0; i < (32 + kSigLoaders - 1) / kSigLoaders; i++) {
                    const int r = lw + kSigLoaders * i;
                    if (r < 32 && rbase + r < n_rows) cp_async16(&slot[j * 32 + r], base + (rbase + r) * row_bytes + col * esz);
                }
            }
            cp_async_commit();
        };
        for (int64_t t = 0; t < ntiles; t++) {
            // announce tile t - (kSigStages - 1) before waiting for a free
            // stage: the folder waits for the next tile before it releases
            // the current one
            if (t >= kSigStages - 1) {
                cp_async_wait<kSigStages - 2>();  // tiles 0 .. t - 1 issued: tile t - (kSigStages - 1) landed
                __syncwarp();
                bar_arrive_all(sig_full((int)((t - (kSigStages - 1)) % kSigStages)));
            }
            if (t >= kSigStages) bar_sync_all(sig_empty((int)(t % kSigStages)));  // the folder released the stage
            issue(t);
        }
        // hand over the tiles still in flight, oldest first
        const int64_t first = ntiles > kSigStages - 1 ? ntiles - (kSigStages - 1) : 0;
        for (int64_t t = first; t < ntiles; t++) {
            cp_async_wait<0>();
            __syncwarp();
            bar_arrive_all(sig_full((int)(t % kSigStages)));
        }
    } else {
        // Full tiles are folded in groups of eight chunks; the next group
        // (the next tile's first, at a tile's last group, after its FULL
        // barrier) is read into registers before the current group's adds,
        // so the shared-memory latency, long while the loaders' copies land,
        // stays off the add chain.  Lanes past n_rows fold stale slots and
        // store nothing.
        float s = 0.0f;
        const bool mine = rbase + lane < n_rows;
        uint4 cur[8];
        if (full_tiles > 0) {
            bar_sync_all(sig_full(0));
            const uint4 *slot = ring(0);
#pragma unroll
            for (int jj = 0; jj < 8; jj++) cur[jj] = slot[jj * 32 + lane];
        }
        for (int64_t t = 0; t < full_tiles; t++) {
            const uint4 *slot = ring(t);
#pragma unroll
            for (int g = 0; g < kSigChunks / 8; g++) {
                uint4 nxt[8];  // left unset when no full tile follows: cur is not read again then
                if (g + 1 < kSigChunks / 8) {
#pragma unroll
                    for (int jj = 0; jj < 8; jj++) nxt[jj] = slot[((g + 1) * 8 + jj) * 32 + lane];
                } else if (t + 1 < ntiles) {
                    bar_sync_all(sig_full((int)((t + 1) % kSigStages)));
                    if (t + 1 < full_tiles) {
                        const uint4 *ns = ring(t + 1);
#pragma unroll
                        for (int jj = 0; jj < 8; jj++) nxt[jj] = ns[jj * 32 + lane];
                    }
                }
#pragma unroll
                for (int jj = 0; jj < 8; jj++) sigma_fold<SRC>(cur[jj], s);
#pragma unroll
                for (int jj = 0; jj < 8; jj++) cur[jj] = nxt[jj];
            }
            // the loaders wait on this stage only once they are kSigStages tiles ahead
            if (t + kSigStages < ntiles) bar_arrive_all(sig_empty((int)(t % kSigStages)));
        }
        if (full_tiles < ntiles) {  // the row's ragged end: whole chunks only (ne0 is a multiple of 8)
            const int64_t t = full_tiles;
            if (t == 0) bar_sync_all(sig_full(0));  // else synced during the last full tile
            const uint4 *slot = ring(t);
            const int nchunks = (int)((ne0 - t * tile_cols + per_chunk - 1) / per_chunk);
            for (int jj = 0; jj < nchunks; jj++) sigma_fold<SRC>(slot[jj * 32 + lane], s);
            if (t + kSigStages < ntiles) bar_arrive_all(sig_empty((int)(t % kSigStages)));
        }
        if (mine) out[rbase + lane] = s / (float)ne0;
    }
}

cudaError_t launch_row_sigma2(const RowSrc &src, int64_t n_rows, float *out, cudaStream_t st) {
    if (n_rows <= 0) return cudaSuccess;
    const int64_t blocks = (n_rows + 31) / 32;
    auto fn = src.src_type == SHC_SRC_BF16 ? row_sigma2_kernel<SHC_SRC_BF16>
              : src.src_type == SHC_SRC_F16 ? row_sigma2_kernel<SHC_SRC_F16>
                                            : row_sigma2_kernel<SHC_SRC_F32>;
    int per_sm = 1;
    cudaError_t e = resident_blocks((const void *)fn, kSigThreads, kSigSmem, &per_sm);  // raises the smem limit
    if (e != cudaSuccess) return e;
    fn<<<(unsigned)blocks, kSigThreads, kSigSmem, st>>>(src, n_rows, out);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Q8_0 (quant.rs:159-169): per 32-block amax, d = amax/127, q = round(x/d).
// HBM-bound.  A lane owns one block (32 consecutive elements, 4-8 16-byte
// loads), so the per-block divisions and the f16 store run once per block;
// a warp covers 32 consecutive blocks and writes their 1088 output bytes from
// shared memory with 16-byte stores.  Blocks with a NaN or infinite element
// or an infinite 1/d take the general rounding path (NaN -> 0, saturating
// clamp); otherwise |x/d| <= 127 (1 + 2^-23)^2 and the code is the magnitude
// rounded half up, sign applied in two's complement.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float max_nan(float a, float b) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}

//
// FUSE: the fused error table (fuse.cuh): warps 0-6 encode a row's 256-element
// unit each (lanes 0-7, one block per lane), warp 7 folds.
template <bool FUSE>
__global__ void __launch_bounds__(256, 4) enc_q8_0_kernel(EncArgs a) {
    constexpr int NWE = 7;
    __shared__ __align__(16) uint8_t s_out[8][32 * 34];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int64_t bpr = a.src.ne0 >> 5;
    const int64_t nblk = a.n_rows * bpr;
    const int64_t nwi = (nblk + 31) >> 5;
    const bool contiguous = a.src.row_stride == a.src.ne0;
    uint8_t *so = s_out[wid];
    extern __shared__ __align__(16) uint8_t q8_fuse_smem[];
    FuseSmem<NWE> *F = reinterpret_cast<FuseSmem<NWE> *>(q8_fuse_smem);
    const int64_t upr = (bpr + 7) >> 3;
    if constexpr (FUSE) {
        fuse_setup(*F);
        if (wid == NWE) {
            fuse_fold(*F, a, upr, lane);
            return;
        }
    }
    // blocks [blk0, blk0 + nb) of the tensor, one per lane
    auto unit = [&](int64_t blk0, int nb) {
        const int64_t blk = blk0 + lane;
        float v[32];
        if (lane < nb) {
            int64_t row = 0, col = blk * 32;  // rows back to back: the block index is the element offset / 32
            if (!contiguous) {
                row = blk / bpr;
                col = (blk - row * bpr) * 32;
            }
#pragma unroll
            for (int m = 0; m < 4; m++) load8(a.src, row, col + m * 8, &v[m * 8]);
        } else {
#pragma unroll
            for (int k = 0; k < 32; k++) v[k] = 0.0f;
        }
        // the NaN-propagating max of |x| flags the blocks that need the
        // general path; without NaN it is the reference's NaN-ignoring max
        float amaxn = 0.0f;
#pragma unroll
        for (int k = 0; k < 32; k++) amaxn = max_nan(amaxn, fabsf(v[k]));
        float amax = amaxn;
        if (!(amaxn < INFINITY)) {
            amax = 0.0f;
#pragma unroll
            for (int k = 0; k < 32; k++) amax = fmaxf(amax, fabsf(v[k]));
        }
        const float d = amax / 127.0f;
        const float id = d > 0.0f ? 1.0f / d : 0.0f;
        uint32_t w[8];
        if (amaxn < INFINITY && id < INFINITY) {
            // two elements per instruction: |y| = |x| id; 2^23 + round-half-up(|y|)
            // by an RZ and an RD add (identities of floor_half_up), the
            // magnitude back out exactly, the sign of x put on it, and the
            // int8 code read as the low byte of m + 1.5 * 2^23
            const float2 id2 = make_float2(id, id);
#pragma unroll
            for (int m = 0; m < 8; m++) {
                uint32_t q[4];
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const float x0 = v[m * 4 + 2 * h], x1 = v[m * 4 + 2 * h + 1];
                    const float2 y = __fmul2_rn(make_float2(fabsf(x0), fabsf(x1)), id2);
                    const float2 u = __fadd2_rd(__fadd2_rz(y, make_float2(0.5f, 0.5f)), make_float2(8388608.0f, 8388608.0f));
                    const float2 r = __fadd2_rn(u, make_float2(-8388608.0f, -8388608.0f));
                    const float2 sgn = make_float2(
                        __uint_as_float(__float_as_uint(r.x) | (__float_as_uint(x0) & 0x80000000u)),
                        __uint_as_float(__float_as_uint(r.y) | (__float_as_uint(x1) & 0x80000000u)));
                    const float2 c = __fadd2_rn(sgn, make_float2(12582912.0f, 12582912.0f));
                    q[2 * h] = __float_as_uint(c.x);
                    q[2 * h + 1] = __float_as_uint(c.y);
                }
                w[m] = __byte_perm(__byte_perm(q[0], q[1], 0x0040), __byte_perm(q[2], q[3], 0x0040), 0x5410);
            }
        } else {
#pragma unroll
            for (int m = 0; m < 8; m++) {
                uint32_t word = 0;
#pragma unroll
                for (int t = 0; t < 4; t++) {
                    // the int8 code is the low byte of r + 1.5 * 2^23 (exact for |r| <= 127)
                    const float r = round_clamp_f(v[m * 4 + t] * id, -127.0f, 127.0f);
                    word |= (__float_as_uint(__fadd_rn(r, 12582912.0f)) & 0xFFu) << (8 * t);
                }
                w[m] = word;
            }
        }
        // 34 bytes per lane at 34 * lane (2-byte aligned): f16 d, then the codes
        uint16_t *o16 = reinterpret_cast<uint16_t *>(so + 34 * lane);
        o16[0] = f16_bits(d);
#pragma unroll
        for (int m = 0; m < 8; m++) {
            o16[1 + 2 * m] = (uint16_t)(w[m] & 0xFFFFu);
            o16[2 + 2 * m] = (uint16_t)(w[m] >> 16);
        }
        __syncwarp();
        if constexpr (!FUSE) store_block(a.dst + blk0 * 34, so, nb * 34, a.dst_aligned16 && nb == 32, lane);
        __syncwarp();
    };
    if constexpr (!FUSE) {
        for (int64_t it = (int64_t)blockIdx.x * 8 + wid; it < nwi; it += (int64_t)gridDim.x * 8) {
            const int64_t left = nblk - (it << 5);
            unit(it << 5, (int)(left < 32 ? left : 32));
        }
    } else {
        FuseIter<NWE> it(a, upr, wid);
        uint32_t fk = 0;
        while (it.next()) {
            const int64_t left = bpr - it.unit * 8;
            if (it.valid) unit(it.row * bpr + it.unit * 8, (int)(left < 8 ? left : 8));
            fuse_emit<SHC_TYPE_Q8_0, 34>(*F, wid, fk, it.valid, a, it.row, it.unit, so, lane);
        }
    }
}

// ceil(t) for 0 <= t <= 2^22 as an int, without the conversion pipe: RU(t +
// 2^23) is 2^23 + ceil(t), whose low mantissa bits are the result.
__device__ __forceinline__ int ceil_small(float t) {
    return (int)(__float_as_uint(__fadd_ru(t, 8388608.0f)) & 0x7FFFFFu);
}


// ---------------------------------------------------------------------------
// Q6_K (quant.rs:231-291) with make_qx_quants(nmax=32) (quant.rs:34-73) per
// 16-element sub-block, and Q3_K (ggml block_q3_K layout) with nmax 4, 6-bit
// signed scale codes and 3-bit levels split into a high-bit mask and 2-bit
// planes.  A warp per super-block; the candidate grids that differ from
// their predecessor are dealt over the lanes and the selection chain is
// replayed serially from shared memory.
// ---------------------------------------------------------------------------
// Per-warp workspace of the make_qx_quants kernel.
struct __align__(16) Qx16Warp {
    float x[16 * 20];       // sub-block s at 20 s (16-byte aligned rows)
    float w[16 * 20];
    float wx[16 * 20];
    float tab[16][20];      // |iscale| of grids t = is + 9 = 0..18
    float2 cand[16][20];    // (sumlx, suml2) of evaluated grids
    float scale[16];
    float mx[16];
    unsigned int mask[16];  // evaluated grids; bit 31: finite sub-block
    uint16_t jobs[16 * 19 + 8];
    uint8_t out[224];
    uint8_t l[256];
};

// make_qx_quants (quant.rs:34-73) with repeated grids skipped: |iscale_t| =
// (nmax + 0.1 (t - 9))/|max| is non-decreasing in t, so |l_i(t)| =
// min(round(|iscale_t x_i|), nmax - 1 or nmax by the sign of iscale*x) is
// non-decreasing with a fixed sign, and grid t repeats grid t-1's levels
// unless an element crosses a threshold k - 1/2 in between (at most two per
// element: |y| spans 1.8 |x|/|max|). A repeated candidate has the same
// (sumlx, suml2) as the one before it, and the selection chain keeps its
// state whether or not it accepts it, so only marked grids are evaluated:
// the exact levels at grids 0 and 18 count the crossings and the estimate
// t ~ 10 (thr |max|/|x| - nmax) + 9, good to well within 0.01 of a grid,
// places each one. The (sub-block, grid) jobs are dealt over the 32 lanes.
//
// FUSE: the fused error table (fuse.cuh), 16 warps: warps 0-14 encode, warp
// 15 folds (one resident block per SM keeps the encoders' count while a
// launch of few rows still spreads over the SMs).
template <int NMAX, bool FUSE>
__global__ void __launch_bounds__(FUSE ? 512 : 256, FUSE ? 1 : 3) enc_qx16_kernel(EncArgs a) {
    constexpr float FN = (float)NMAX;
    constexpr int OUT = NMAX == 32 ? 210 : 110;
    constexpr int NWE = 15;
    extern __shared__ __align__(16) uint8_t qx16_smem[];
    const int wid = threadIdx.x >> 5;
    Qx16Warp *W = reinterpret_cast<Qx16Warp *>(qx16_smem) + wid;
    const int lane = threadIdx.x & 31;
    const int s = lane >> 1, q = lane & 1;
    const int64_t ne0 = a.src.ne0, nsb = ne0 >> 8, total = a.n_rows * nsb;
    FuseSmem<NWE> *F = reinterpret_cast<FuseSmem<NWE> *>(qx16_smem + NWE * sizeof(Qx16Warp));
    if constexpr (FUSE) {
        fuse_setup(*F);
        if (wid == NWE) {
            fuse_fold(*F, a, nsb, lane);
            return;
        }
    }
    auto unit = [&](int64_t g) {
        const int64_t row = g / nsb;
        const int64_t sbi = g - row * nsb;
        const int64_t col0 = sbi << 8;
        const float sig = a.sigma2[row];
        const float *imr = im_row(a.im, ne0, a.row0 + row * a.row_step);
        float v[8], base[8];
        load8(a.src, row, col0 + lane * 8, v);
        load_im8(imr, col0 + lane * 8, base);
        {
            float wk[8];
#pragma unroll
            for (int k = 0; k < 8; k++) wk[k] = base[k] * sqrtf(sig + v[k] * v[k]);
            float4 *px = reinterpret_cast<float4 *>(&W->x[s * 20 + q * 8]);
            float4 *pw = reinterpret_cast<float4 *>(&W->w[s * 20 + q * 8]);
            float4 *pwx = reinterpret_cast<float4 *>(&W->wx[s * 20 + q * 8]);
            px[0] = make_float4(v[0], v[1], v[2], v[3]);
            px[1] = make_float4(v[4], v[5], v[6], v[7]);
            pw[0] = make_float4(wk[0], wk[1], wk[2], wk[3]);
            pw[1] = make_float4(wk[4], wk[5], wk[6], wk[7]);
            pwx[0] = make_float4(wk[0] * v[0], wk[1] * v[1], wk[2] * v[2], wk[3] * v[3]);
            pwx[1] = make_float4(wk[4] * v[4], wk[5] * v[5], wk[6] * v[6], wk[7] * v[7]);
        }
        // max |x| of the sub-block, first strict maximum (quant.rs:38-44)
        float amax = 0.0f, mx = 0.0f;
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const float av = fabsf(v[k]);
            if (av > amax) { amax = av; mx = v[k]; }
        }
        {
            const float oa = __shfl_xor_sync(0xffffffffu, amax, 1), om = __shfl_xor_sync(0xffffffffu, mx, 1);
            if (q == 0 ? oa > amax : !(amax > oa)) { amax = oa; mx = om; }
        }
        const bool live = !(amax < kGroupMaxEps);
        // with finite inputs iscale*x is finite, so the NaN -> 0 rule of the
        // saturating cast cannot trigger and the plain clamp is exact
        float xsum = 0.0f;
#pragma unroll
        for (int k = 0; k < 8; k++) xsum += v[k] * 0.0f;
        xsum += __shfl_xor_sync(0xffffffffu, xsum, 1);
        const bool finite = xsum == 0.0f;
        if (live) {
            for (int t = q; t < 19; t += 2) W->tab[s][t] = fabsf(-(FN + 0.1f * (float)(t - 9)) / mx);
        }
        __syncwarp();
        unsigned int mask = 0;
        if (live && finite) {
            const float t0 = W->tab[s][0], t18 = W->tab[s][18];
            const float amx = fabsf(mx);
            mask = 1u;
#pragma unroll 1
            for (int k = 0; k < 8; k++) {
                const float xv = W->x[s * 20 + q * 8 + k];
                const float ax = fabsf(xv);
                // iscale*x > 0 (sign of x differs from max's) clamps at nmax - 1
                const float cap = (xv != 0.0f && (signbit(xv) != signbit(mx))) ? FN - 1.0f : FN;
                const float m0 = fminf(floor_half_up(__fmul_rn(t0, ax)), cap);
                const float m18 = fminf(floor_half_up(__fmul_rn(t18, ax)), cap);
                if (m18 > m0) {
                    const float ru = amx / ax;
#pragma unroll
                    for (int c = 1; c <= 2; c++) {
                        const float thr = m0 + ((float)c - 0.5f);
                        if (thr < m18) {
                            const float z = 10.0f * (thr * ru - FN) + 9.0f;
                            mask |= 1u << ceil_small(fminf(fmaxf(z - 0.01f, 0.5f), 18.0f));
                            mask |= 1u << ceil_small(fminf(fmaxf(z + 0.01f, 0.5f), 18.0f));
                        }
                    }
                }
            }
        } else if (live) {
            mask = (1u << 19) - 1;
        }
        mask |= __shfl_xor_sync(0xffffffffu, mask, 1);
        // job list: lane q lists the grids among bits [10 q, 10 q + 10)
        const int cnt = __popc(mask);
        int incl = q == 0 ? cnt : 0;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, incl, off);
            if (lane >= off) incl += t;
        }
        const int njobs = __shfl_sync(0xffffffffu, incl, 31);
        {
            int pos = __shfl_sync(0xffffffffu, incl, lane - q) - cnt + (q ? __popc(mask & 0x3FFu) : 0);
            unsigned int bits = q ? (mask >> 10) : (mask & 0x3FFu);
            while (bits != 0) {
                W->jobs[pos++] = (uint16_t)((s << 8) | ((q ? 10 : 0) + __ffs(bits) - 1));
                bits &= bits - 1;
            }
        }
        if (q == 0) {
            W->mask[s] = mask | (finite ? 0x80000000u : 0u);
            W->mx[s] = mx;
        }
        __syncwarp();
        // (sumlx, suml2) of the listed grids (quant.rs:48-63)
#pragma unroll 1
        for (int jj = lane; jj < njobs; jj += 32) {
            const int code = W->jobs[jj];
            const int js = code >> 8, t = code & 0xFF;
            float x[16], w[16], wx[16];
#pragma unroll
            for (int i = 0; i < 16; i += 4) {
                const float4 a4 = *reinterpret_cast<const float4 *>(&W->x[js * 20 + i]);
                const float4 b4 = *reinterpret_cast<const float4 *>(&W->w[js * 20 + i]);
                const float4 c4 = *reinterpret_cast<const float4 *>(&W->wx[js * 20 + i]);
                x[i] = a4.x; x[i + 1] = a4.y; x[i + 2] = a4.z; x[i + 3] = a4.w;
                w[i] = b4.x; w[i + 1] = b4.y; w[i + 2] = b4.z; w[i + 3] = b4.w;
                wx[i] = c4.x; wx[i + 1] = c4.y; wx[i + 2] = c4.z; wx[i + 3] = c4.w;
            }
            // -(nmax + 0.1 is)/max: the magnitude from the table, the sign of -max
            const float iscale = copysignf(W->tab[js][t], -W->mx[js]);
            float sumlx = 0.0f, suml2 = 0.0f;
            if (W->mask[js] & 0x80000000u) {
                const float2 is2 = make_float2(iscale, iscale);
#pragma unroll
                for (int i = 0; i < 16; i += 2) {
                    const float2 y = __fmul2_rn(is2, make_float2(x[i], x[i + 1]));
                    const float2 r = floor_half_up2(make_float2(fabsf(y.x), fabsf(y.y)));
                    const float2 l = make_float2(fminf(fmaxf(copysignf(r.x, y.x), -FN), FN - 1.0f),
                                                 fminf(fmaxf(copysignf(r.y, y.y), -FN), FN - 1.0f));
                    const float2 lx = __fmul2_rn(make_float2(wx[i], wx[i + 1]), l);
                    const float2 l2 = __fmul2_rn(make_float2(w[i], w[i + 1]), __fmul2_rn(l, l));
                    sumlx = __fadd_rn(sumlx, lx.x);
                    suml2 = __fadd_rn(suml2, l2.x);
                    sumlx = __fadd_rn(sumlx, lx.y);
                    suml2 = __fadd_rn(suml2, l2.y);
                }
            } else {
#pragma unroll
                for (int i = 0; i < 16; i++) {
                    const float l = round_clamp_f(iscale * x[i], -FN, FN - 1.0f);
                    sumlx += wx[i] * l;
                    suml2 += w[i] * (l * l);
                }
            }
            W->cand[js][t] = make_float2(sumlx, suml2);
        }
        __syncwarp();
        // the selection chain (quant.rs:64-70) over the evaluated grids
        if (q == 0) {
            float best_scale = 0.0f, best = 0.0f;
            bool first = true;
            unsigned int m = mask;
            while (m != 0) {
                const int c = __ffs(m) - 1;
                m &= m - 1;
                const float2 cs = W->cand[s][c];
                if (cs.y > 0.0f && (first || cs.x * cs.x > best * cs.y)) {
                    const float sc = cs.x / cs.y;
                    best_scale = sc;
                    best = sc * cs.x;
                    first = false;
                }
            }
            W->scale[s] = best_scale;
        }
        __syncwarp();
        // largest |scale| over the 16 sub-blocks, first strict maximum
        // (quant.rs:243-246): lanes 2s and 2s+1 hold sub-block s; a butterfly
        // keeps the lower sub-block's value unless the higher one's is
        // strictly larger (NaN and zero never replace the initial 0)
        const float best_scale = W->scale[s];
        float max_abs = 0.0f, max_scale = 0.0f;
        if (fabsf(best_scale) > 0.0f) { max_abs = fabsf(best_scale); max_scale = best_scale; }
#pragma unroll
        for (int off = 2; off <= 16; off <<= 1) {
            const float oa = __shfl_xor_sync(0xffffffffu, max_abs, off), om = __shfl_xor_sync(0xffffffffu, max_scale, off);
            if ((lane & off) == 0 ? oa > max_abs : !(max_abs > oa)) { max_abs = oa; max_scale = om; }
        }
        uint8_t *o = W->out;
        if (max_abs < kGroupMaxEps) {
            for (int i = lane; i < OUT; i += 32) o[i] = 0;
        } else if (NMAX == 32) {  // Q6_K (quant.rs:258-290)
            const float iscale = -128.0f / max_scale;
            const float d = 1.0f / iscale;
            const int8_t qsc = (int8_t)(uint8_t)(min(nearest_int(iscale * best_scale), 127) & 0xFF);
            const float dd = d * (float)qsc;
            // lane owns elements lane*8..lane*8+7 = sub-block s, offset q*8
#pragma unroll
            for (int k = 0; k < 8; k++) {
                const int l = dd == 0.0f ? 32 : (int)round_clamp_f(v[k] / dd, -32.0f, 31.0f) + 32;
                W->l[lane * 8 + k] = (uint8_t)l;
            }
            if (q == 0) o[192 + s] = (uint8_t)qsc;
            if (lane == 0) {
                const uint16_t h = f16_bits(d);
                o[208] = (uint8_t)(h & 0xFF);
                o[209] = (uint8_t)(h >> 8);
            }
            __syncwarp();
            const uint8_t *L = W->l;
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const uint8_t *lo = L + h * 128;
                const int l = lane;
                o[h * 64 + l] = (uint8_t)((lo[l] & 0xF) | ((lo[l + 64] & 0xF) << 4));
                o[h * 64 + 32 + l] = (uint8_t)((lo[l + 32] & 0xF) | ((lo[l + 96] & 0xF) << 4));
                o[128 + h * 32 + l] = (uint8_t)((lo[l] >> 4) | ((lo[l + 32] >> 4) << 2) | ((lo[l + 64] >> 4) << 4) |
                                                ((lo[l + 96] >> 4) << 6));
            }
        } else {  // Q3_K: 6-bit signed scale codes, 3-bit levels (hmask + 2-bit planes)
            const float iscale = -32.0f / max_scale;
            const float d = 1.0f / iscale;
            const int qsc = (int)round_clamp_f(iscale * best_scale, -32.0f, 31.0f);
            const float dd = d * (float)qsc;
#pragma unroll
            for (int k = 0; k < 8; k++) {
                const int l = dd == 0.0f ? 4 : (int)round_clamp_f(v[k] / dd, -4.0f, 3.0f) + 4;
                W->l[lane * 8 + k] = (uint8_t)l;
            }
            // scale codes u = qsc + 32 of every sub-block, from its even lane
            const int u = qsc + 32;
            const int ua = __shfl_sync(0xffffffffu, u, 2 * (lane & 7));           // sub-block lane & 7
            const int ub = __shfl_sync(0xffffffffu, u, 2 * ((lane & 7) + 8));     // sub-block (lane & 7) + 8
            const int uc[4] = {__shfl_sync(0xffffffffu, u, 2 * ((lane & 3) + 0)), __shfl_sync(0xffffffffu, u, 2 * ((lane & 3) + 4)),
                               __shfl_sync(0xffffffffu, u, 2 * ((lane & 3) + 8)), __shfl_sync(0xffffffffu, u, 2 * ((lane & 3) + 12))};
            if (lane < 8) o[96 + lane] = (uint8_t)((ua & 0xF) | ((ub & 0xF) << 4));
            if (lane >= 8 && lane < 12)
                o[104 + (lane & 3)] = (uint8_t)(((uc[0] >> 4) & 3) | (((uc[1] >> 4) & 3) << 2) | (((uc[2] >> 4) & 3) << 4) |
                                                (((uc[3] >> 4) & 3) << 6));
            if (lane == 0) {
                const uint16_t h = f16_bits(d);
                o[108] = (uint8_t)(h & 0xFF);
                o[109] = (uint8_t)(h >> 8);
            }
            __syncwarp();
            const uint8_t *L = W->l;
            uint8_t hm = 0;  // hmask byte `lane`: bit j = high bit of element j*32 + lane
#pragma unroll
            for (int j = 0; j < 8; j++) hm |= (uint8_t)(((L[j * 32 + lane] >> 2) & 1) << j);
            o[lane] = hm;
#pragma unroll
            for (int h = 0; h < 2; h++) {  // qs byte h*32 + lane: elements h*128 + j*32 + lane at bits 2j
                uint8_t b = 0;
#pragma unroll
                for (int j = 0; j < 4; j++) b |= (uint8_t)((L[h * 128 + j * 32 + lane] & 3) << (2 * j));
                o[32 + h * 32 + lane] = b;
            }
        }
        __syncwarp();
        if constexpr (!FUSE) store_block(a.dst + row * a.dst_row_bytes + sbi * OUT, o, OUT, false, lane);
        __syncwarp();
    };
    if constexpr (!FUSE) {
        for (int64_t g = (int64_t)blockIdx.x * 8 + wid; g < total; g += (int64_t)gridDim.x * 8) unit(g);
    } else {
        FuseIter<NWE> it(a, nsb, wid);
        uint32_t fk = 0;
        while (it.next()) {
            if (it.valid) unit(it.row * nsb + it.unit);
            fuse_emit<NMAX == 32 ? SHC_TYPE_Q6_K : SHC_TYPE_Q3_K, 0>(*F, wid, fk, it.valid, a, it.row, it.unit, W->out,
                                                                    lane);
        }
    }
}

// ---------------------------------------------------------------------------
// Q4_K / Q5_K (quant.rs:294-379) and Q2_K with make_qkx3_quants
// (quant.rs:77-141, rmin -0.9, rdelta 0.05, 37 grids) per 32-element (Q4_K,
// Q5_K) or 16-element (Q2_K) sub-block; a warp per super-block.
//
// A lane evaluating a grid reads the sub-block as float2 pairs and runs the element-wise
// products of a grid with packed f32x2 multiplies and adds (two IEEE-rounded
// f32 operations per instruction, the same results as scalar code); the
// reference's running sums stay scalar and in element order.  x is kept
// negated (nx = -x): x - vmin = -(nx + vmin), w*l*x = -((w*l)*nx) and
// diff - x = diff + nx are exact identities of round-to-nearest, so every
// rounded value equals the reference's.
// ---------------------------------------------------------------------------
// NG grids of make_qkx3_quants over the lane's 32 elements (quant.rs:109-118),
// interleaved element by element so that their serial sums form independent
// dependency chains: l = nearest_int(iscale * (x - vmin)).clamp(0, nmax) and
// the three weighted sums per grid.  CLEAN: every iscale and (x - vmin) is
// finite, so y = iscale*(x - vmin) is >= 0 or +inf and the clamp at 0 is not
// needed.
template <bool CLEAN, int NG, int NP>
__device__ __forceinline__ void qkx3_grids(const float *snx, const float *sw, const float *su, const float (&iscale)[NG],
                                           float fn, float2 (&l)[NG][NP], float (&sl)[NG], float (&sl2)[NG],
                                           float (&sxl)[NG]) {
    float2 nis[NG];
#pragma unroll
    for (int g = 0; g < NG; g++) {
        nis[g] = make_float2(-iscale[g], -iscale[g]);
        sl[g] = 0.0f;
        sl2[g] = 0.0f;
        sxl[g] = 0.0f;
    }
#pragma unroll
    for (int i = 0; i < NP; i++) {
        const float4 n4 = reinterpret_cast<const float4 *>(snx)[i >> 1];
        const float4 w4 = reinterpret_cast<const float4 *>(sw)[i >> 1];
        const float2 nxi = (i & 1) ? make_float2(n4.z, n4.w) : make_float2(n4.x, n4.y);
        const float2 wi = (i & 1) ? make_float2(w4.z, w4.w) : make_float2(w4.x, w4.y);
        const float4 u4 = reinterpret_cast<const float4 *>(su)[i >> 1];
        const float2 ui = (i & 1) ? make_float2(u4.z, u4.w) : make_float2(u4.x, u4.y);  // -(x - vmin)
#pragma unroll
        for (int g = 0; g < NG; g++) {
            const float2 r = floor_half_up2(__fmul2_rn(nis[g], ui));  // the first add is RZ
            float2 li;
            if (CLEAN) {
                li = make_float2(fminf(r.x, fn), fminf(r.y, fn));
            } else {
                li = make_float2(fminf(fmaxf(r.x, 0.0f), fn), fminf(fmaxf(r.y, 0.0f), fn));
            }
            l[g][i] = li;
            const float2 wl = __fmul2_rn(wi, li);
            const float2 wll = __fmul2_rn(wi, __fmul2_rn(li, li));  // (l*l) is exact, as the integer product
            const float2 nwlx = __fmul2_rn(wl, nxi);                // -(w*l*x)
            sl[g] = __fadd_rn(sl[g], wl.x);
            sl2[g] = __fadd_rn(sl2[g], wll.x);
            sxl[g] = __fsub_rn(sxl[g], nwlx.x);
            sl[g] = __fadd_rn(sl[g], wl.y);
            sl2[g] = __fadd_rn(sl2[g], wll.y);
            sxl[g] = __fsub_rn(sxl[g], nwlx.y);
        }
    }
}

// Weighted squared error of NG candidate (scale, min) fits, interleaved
// (quant.rs:125-128 and 100-101): diff = scale*l + min - x, err += w*diff*diff.
template <int NG, int NP>
__device__ __forceinline__ void qkx3_errors(const float *snx, const float *sw, const float2 (&l)[NG][NP],
                                            const float (&ts)[NG], const float (&tm)[NG], float (&err)[NG]) {
#pragma unroll
    for (int g = 0; g < NG; g++) err[g] = 0.0f;
#pragma unroll
    for (int i = 0; i < NP; i++) {
        const float4 n4 = reinterpret_cast<const float4 *>(snx)[i >> 1];
        const float4 w4 = reinterpret_cast<const float4 *>(sw)[i >> 1];
        const float2 nxi = (i & 1) ? make_float2(n4.z, n4.w) : make_float2(n4.x, n4.y);
        const float2 wi = (i & 1) ? make_float2(w4.z, w4.w) : make_float2(w4.x, w4.y);
#pragma unroll
        for (int g = 0; g < NG; g++) {
            const float2 p = __fmul2_rn(make_float2(ts[g], ts[g]), l[g][i]);
            const float2 d = __fadd2_rn(make_float2(__fadd_rn(p.x, tm[g]), __fadd_rn(p.y, tm[g])), nxi);
            const float2 e = __fmul2_rn(__fmul2_rn(wi, d), d);
            err[g] = __fadd_rn(err[g], e.x);
            err[g] = __fadd_rn(err[g], e.y);
        }
    }
}

// make_qkx3_quants over a whole super-block per warp, with duplicate grids
// skipped.  For u = x - vmin >= 0 the grid scales iscale_j = (rmin + rdelta*j
// + nmax)/(vmax - vmin) are non-decreasing in j (each rounded step is
// monotone), so every level l_i(j) = min(round(iscale_j * u_i), nmax) is
// non-decreasing in j, and the level vector of grid j equals that of grid
// j-1 unless some element crosses a rounding threshold k - 1/2 between them.
// Equal level vectors give equal sums, (scale, min) and error, so such a
// grid never replaces the earlier one under the reference's strict `<`
// (quant.rs:129): only grids where some element may cross are evaluated.
// y_36 - y_0 = 1.8 u / (vmax - vmin) <= 1.8 (plus rounding), so an element
// crosses at most two thresholds (round half away from zero of y >= 0 is
// floor(y + 1/2), so l_i(j) >= k iff y_j >= k - 1/2); the exact levels at
// grids 0 and 36 count them and a bounded estimate places them.  Sub-blocks
// with a non-finite range or scale evaluate every grid.
//
// The distinct (sub-block, grid) jobs of the warp's super-block, plus each
// sub-block's initial nmax/(vmax-vmin) grid, are listed in shared memory in
// (sub-block, grid) order and dealt to the 32 lanes round by round; a
// sub-block's best (error, grid) is kept with a 64-bit shared-memory
// atomicMin on (order-preserving error bits, grid), which keeps the first
// minimum as the reference's chain does.
template <int N>
struct __align__(16) Qkx3Warp {
    static constexpr int LPS = N / 8;    // lanes per sub-block (8 elements each)
    static constexpr int NSB = 256 / N;  // sub-blocks per super-block
    static constexpr int PAD = N + 4;    // float stride of a staged sub-block
    float4 par[NSB];                     // sum_w, sum_x, vmin, nmax/(vmax-vmin)
    float nx[NSB * PAD];                 // -x
    float w[NSB * PAD];                  // element weights
    float u[NSB * PAD];                  // -(x - vmin)
    float isc[NSB][40];                  // iscale of grids 0..36
    float ts[NSB][38];                   // (scale, min) of evaluated grids
    float tm[NSB][38];
    float init_err[NSB];
    float2 par2[NSB];                    // 1/iscale0, clean
    unsigned long long best[NSB];
    uint16_t jobs[NSB * 38];             // (sub-block << 8) | grid
    uint8_t out[176];
    uint8_t l[256];
};

__device__ __forceinline__ unsigned int err_key(float e) {
    const unsigned int b = __float_as_uint(e);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float err_from_key(unsigned int k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}


// FUSE: the fused error table (fuse.cuh), 16 warps (Q2_K, whose workspace is
// larger: 8): the last warp folds, the others encode.
constexpr int kQkx3Warps = 8;
template <int N, int NMAX, bool FUSE>
__device__ __forceinline__ void qkx3_super_blocks(const EncArgs &a, uint8_t *smem) {
    using Wp = Qkx3Warp<N>;
    constexpr int LPS = Wp::LPS, PAD = Wp::PAD;
    constexpr float FN = (float)NMAX;
    constexpr bool Q2 = N == 16;
    constexpr int BB = Q2 ? 84 : (NMAX == 31 ? 176 : 144);
    constexpr int NWE = Q2 ? 7 : 15;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    Wp *W = reinterpret_cast<Wp *>(smem) + wid;
    const int s = lane / LPS, q = lane % LPS;
    const int64_t ne0 = a.src.ne0, nsb = ne0 >> 8, total = a.n_rows * nsb;
    const int64_t nwarps = (int64_t)gridDim.x * kQkx3Warps;
    FuseSmem<NWE> *F = reinterpret_cast<FuseSmem<NWE> *>(smem + NWE * sizeof(Wp));
    if constexpr (FUSE) {
        fuse_setup(*F);
        if (wid == NWE) {
            fuse_fold(*F, a, nsb, lane);
            return;
        }
    }
    float *snx = &W->nx[s * PAD];
    float *sw = &W->w[s * PAD];
    float *su = &W->u[s * PAD];
    auto unit = [&](int64_t g) {
        const int64_t row = g / nsb;
        const int64_t sbi = g - row * nsb;
        const int64_t col0 = sbi << 8;
        const float sig = a.sigma2[row];
        const float *imr = im_row(a.im, ne0, a.row0 + row * a.row_step);
        float v[8], base[8];
        load8(a.src, row, col0 + lane * 8, v);
        load_im8(imr, col0 + lane * 8, base);
        // element weights (quant.rs:144-151): base * sqrt(sigma2 + x*x)
        {
            float wk[8];
#pragma unroll
            for (int k = 0; k < 8; k += 2) {
                const float2 vv = make_float2(v[k], v[k + 1]);
                const float2 vv2 = __fmul2_rn(vv, vv);
                const float2 sq = make_float2(sqrtf(__fadd_rn(sig, vv2.x)), sqrtf(__fadd_rn(sig, vv2.y)));
                const float2 ww = __fmul2_rn(make_float2(base[k], base[k + 1]), sq);
                wk[k] = ww.x;
                wk[k + 1] = ww.y;
            }
            float4 *pn = reinterpret_cast<float4 *>(snx + q * 8);
            float4 *pw = reinterpret_cast<float4 *>(sw + q * 8);
            pn[0] = make_float4(-v[0], -v[1], -v[2], -v[3]);
            pn[1] = make_float4(-v[4], -v[5], -v[6], -v[7]);
            pw[0] = make_float4(wk[0], wk[1], wk[2], wk[3]);
            pw[1] = make_float4(wk[4], wk[5], wk[6], wk[7]);
        }
        // vmin/vmax folds (quant.rs:87-88) are order-independent (NaN is
        // skipped): this lane's 8 values, then the lanes of the sub-block.
        // The sign of a zero vmin/vmax never reaches the bytes (it only
        // enters x - vmin, scale*l + vmin, and -vmin folded with +0 by max).
        float vmin, vmax;
        {
            float mn = fminf(fminf(fminf(v[0], v[1]), fminf(v[2], v[3])), fminf(fminf(v[4], v[5]), fminf(v[6], v[7])));
            float mx = fmaxf(fmaxf(fmaxf(v[0], v[1]), fmaxf(v[2], v[3])), fmaxf(fmaxf(v[4], v[5]), fmaxf(v[6], v[7])));
#pragma unroll
            for (int off = 1; off < LPS; off <<= 1) {
                mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, off));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            }
            vmin = fminf(fminf(INFINITY, mn), 0.0f);
            vmax = fmaxf(-INFINITY, mx);
        }
        const bool degen = vmax <= vmin;
        const float range = vmax - vmin;
        {
            // u = nx + vmin = -(x - vmin): the same rounded value for every grid
            float4 *pu = reinterpret_cast<float4 *>(su + q * 8);
            pu[0] = make_float4(__fadd_rn(-v[0], vmin), __fadd_rn(-v[1], vmin), __fadd_rn(-v[2], vmin),
                                __fadd_rn(-v[3], vmin));
            pu[1] = make_float4(__fadd_rn(-v[4], vmin), __fadd_rn(-v[5], vmin), __fadd_rn(-v[6], vmin),
                                __fadd_rn(-v[7], vmin));
            // iscale of the 37 grids (quant.rs:108), split over the sub-block's lanes
            for (int j = q; j < 37; j += LPS) W->isc[s][j] = (-0.9f + 0.05f * (float)j + FN) / range;
        }
        __syncwarp();
        const float iscale0 = FN / range;
        const float scale0 = 1.0f / iscale0;
        const bool clean = !degen && range < INFINITY && W->isc[s][36] < INFINITY;
        // grids whose level vector may differ from the previous grid's: a
        // superset of the crossing grids (evaluating a repeated grid changes
        // nothing), from the estimate j ~ 20 (thr (vmax-vmin)/u - (nmax-0.9)).
        // Its error against the first grid with iscale_j*u >= thr is below
        // 5e-4 grid steps (rounding of iscale_j, the product and the estimate,
        // 2-ulp quotient for normal u), so every integer in
        // [ceil(z - 0.004), ceil(z + 0.004)] (one or two grids) is marked.
        unsigned long long mask = 0;
        if (!degen) {
            if (clean) {
                const float i0 = W->isc[s][0], i36 = W->isc[s][36];
                uint32_t mlo = 1u, mhi = 0u;  // grids 0-31 and 32-36
#pragma unroll 1
                for (int k = 0; k < 8; k++) {
                    const float uk = -su[q * 8 + k];  // x - vmin
                    const float l0 = fminf(floor_half_up(__fmul_rn(i0, uk)), FN);
                    const float l36 = fminf(floor_half_up(__fmul_rn(i36, uk)), FN);
                    if (l36 > l0) {
                        if (uk >= 1.17549435e-38f && uk <= 8.50705917e37f) {
                            const float ru = __fdividef(range, uk);
#pragma unroll
                            for (int c = 1; c <= 2; c++) {
                                const float thr = l0 + ((float)c - 0.5f);
                                if (thr < l36) {
                                    const float z = 20.0f * (thr * ru - (FN - 0.9f));
                                    const int jl = ceil_small(fminf(fmaxf(z - 0.004f, 0.5f), 36.0f));
                                    const int jh = ceil_small(fminf(fmaxf(z + 0.004f, 0.5f), 36.0f));
                                    if (jl < 32) mlo |= 1u << jl;
                                    else mhi |= 1u << (jl - 32);
                                    if (jh < 32) mlo |= 1u << jh;
                                    else mhi |= 1u << (jh - 32);
                                }
                            }
                        } else {  // subnormal or huge u: no usable estimate
                            mlo = ~0u;
                            mhi = 0x1Fu;
                        }
                    }
                }
                mask = ((unsigned long long)mhi << 32) | mlo;
            } else {
                mask = (1ull << 37) - 1;
            }
            mask |= 1ull << 37;  // the initial grid
        }
#pragma unroll
        for (int off = 1; off < LPS; off <<= 1) mask |= __shfl_xor_sync(0xffffffffu, mask, off);
        // job list: exclusive prefix of the sub-blocks' job counts; lane q of
        // a sub-block lists the grids among bits [q*B, q*B + B) of its mask
        const int cnt = __popcll(mask);
        int incl = q == 0 ? cnt : 0;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, incl, off);
            if (lane >= off) incl += t;
        }
        const int njobs = __shfl_sync(0xffffffffu, incl, 31);
        {
            constexpr int B = (38 + LPS - 1) / LPS;
            const int lo_bit = q * B;
            int pos = __shfl_sync(0xffffffffu, incl, lane - q) - cnt + __popcll(mask & ((1ull << lo_bit) - 1));
            unsigned int bits = (unsigned int)((mask >> lo_bit) & ((1ull << B) - 1));
            while (bits != 0) {
                W->jobs[pos++] = (uint16_t)((s << 8) | (lo_bit + __ffs(bits) - 1));
                bits &= bits - 1;
            }
        }
        float sum_w = 0.0f, sum_x = 0.0f;
        if (!degen) {
#pragma unroll
            for (int c = 0; c < N / 4; c++) {
                const float4 n4 = reinterpret_cast<const float4 *>(snx)[c];
                const float4 w4 = reinterpret_cast<const float4 *>(sw)[c];
                const float2 p0 = __fmul2_rn(make_float2(w4.x, w4.y), make_float2(n4.x, n4.y));
                const float2 p1 = __fmul2_rn(make_float2(w4.z, w4.w), make_float2(n4.z, n4.w));
                sum_w = __fadd_rn(sum_w, w4.x);
                sum_x = __fsub_rn(sum_x, p0.x);
                sum_w = __fadd_rn(sum_w, w4.y);
                sum_x = __fsub_rn(sum_x, p0.y);
                sum_w = __fadd_rn(sum_w, w4.z);
                sum_x = __fsub_rn(sum_x, p1.x);
                sum_w = __fadd_rn(sum_w, w4.w);
                sum_x = __fsub_rn(sum_x, p1.y);
            }
        }
        if (q == 0) {
            W->par[s] = make_float4(sum_w, sum_x, vmin, iscale0);
            W->par2[s] = make_float2(scale0, clean ? 1.0f : 0.0f);
            W->best[s] = ~0ull;
        }
        __syncwarp();
        // evaluate the listed grids (quant.rs:109-135), one per lane per round
#pragma unroll 1
        for (int t = lane; t < njobs; t += 32) {
            const int code = W->jobs[t];
            const int js = code >> 8, j = code & 0xFF;
            const float4 pa = W->par[js];
            const float2 pb = W->par2[js];
            const float *jnx = &W->nx[js * PAD], *jw = &W->w[js * PAD], *ju = &W->u[js * PAD];
            float isc[1] = {j == 37 ? pa.w : W->isc[js][j]};
            float sl[1], sl2[1], sxl[1];
            float2 l[1][N / 2];
            if (pb.y != 0.0f) qkx3_grids<true, 1, N / 2>(jnx, jw, ju, isc, FN, l, sl, sl2, sxl);
            else qkx3_grids<false, 1, N / 2>(jnx, jw, ju, isc, FN, l, sl, sl2, sxl);
            float ts[1], tm[1];
            bool valid = true;
            if (j == 37) {
                ts[0] = pb.x;
                tm[0] = pa.z;
            } else {
                const float D = __fsub_rn(__fmul_rn(pa.x, sl2[0]), __fmul_rn(sl[0], sl[0]));
                valid = D > 0.0f;
                ts[0] = __fsub_rn(__fmul_rn(pa.x, sxl[0]), __fmul_rn(pa.y, sl[0])) / D;
                tm[0] = __fsub_rn(__fmul_rn(sl2[0], pa.y), __fmul_rn(sl[0], sxl[0])) / D;
                if (tm[0] > 0.0f) {
                    tm[0] = 0.0f;
                    ts[0] = sl2[0] > 0.0f ? sxl[0] / sl2[0] : 0.0f;
                }
            }
            float err[1];
            qkx3_errors<1, N / 2>(jnx, jw, l, ts, tm, err);
            if (j == 37) {
                W->init_err[js] = err[0];
            } else if (valid && err[0] == err[0]) {
                W->ts[js][j] = ts[0];
                W->tm[js][j] = tm[0];
                atomicMin(&W->best[js], ((unsigned long long)err_key(err[0]) << 32) | (unsigned)j);
            }
        }
        __syncwarp();
        float scale, mn;
        {
            const unsigned long long bk = W->best[s];
            const int best_j = bk == ~0ull ? -1 : (int)(bk & 0xFFu);
            if (degen) {
                scale = 0.0f;
                mn = vmin;
            } else if (best_j >= 0 && err_from_key((unsigned)(bk >> 32)) < W->init_err[s]) {
                scale = W->ts[s][best_j];
                mn = W->tm[s][best_j];
            } else {
                scale = scale0;
                mn = vmin;
            }
        }
        const float mins_s = -mn;
        float max_scale = scale, max_min = mins_s;
#pragma unroll
        for (int off = LPS; off <= 16; off <<= 1) {
            max_scale = rmaxf(max_scale, __shfl_xor_sync(0xffffffffu, max_scale, off));
            max_min = rmaxf(max_min, __shfl_xor_sync(0xffffffffu, max_min, off));
        }
        max_scale = rmaxf(0.0f, max_scale);
        max_min = rmaxf(0.0f, max_min);
        constexpr float QS = Q2 ? 15.0f : 63.0f;  // scale/min code range
        const float inv_scale = max_scale > 0.0f ? QS / max_scale : 0.0f;
        const float inv_min = max_min > 0.0f ? QS / max_min : 0.0f;
        const int lsq = (int)round_clamp0_f(inv_scale * scale, QS);
        const int lmq = (int)round_clamp0_f(inv_min * mins_s, QS);
        const float d = max_scale / QS;
        const float dmin = max_min / QS;
        const float dsub = d * (float)lsq;
        const float msub = dmin * (float)lmq;
#pragma unroll
        for (int k = 0; k < 8; k++) {
            // (x + msub) = (msub - nx); x re-read from shared memory
            const int l = dsub == 0.0f ? 0 : (int)round_clamp0_f(__fsub_rn(msub, snx[q * 8 + k]) / dsub, FN);
            W->l[lane * 8 + k] = (uint8_t)l;
        }
        uint8_t *o = W->out;
        const uint8_t *L = W->l;
        if (Q2) {
            // Q2_K: 4-bit scale | min << 4 per sub-block, d/dmin f16 at 80/82
            if (q == 0) o[s] = (uint8_t)(lsq | (lmq << 4));
            if (lane == 0) {
                const uint16_t hd = f16_bits(d), hm = f16_bits(dmin);
                o[80] = (uint8_t)(hd & 0xFF);
                o[81] = (uint8_t)(hd >> 8);
                o[82] = (uint8_t)(hm & 0xFF);
                o[83] = (uint8_t)(hm >> 8);
            }
            __syncwarp();
#pragma unroll
            for (int h = 0; h < 2; h++) {  // qs byte h*32 + lane: elements h*128 + j*32 + lane at bits 2j
                uint8_t b = 0;
#pragma unroll
                for (int j = 0; j < 4; j++) b |= (uint8_t)(L[h * 128 + j * 32 + lane] << (2 * j));
                o[16 + h * 32 + lane] = b;
            }
        } else {
            // 6-bit scale/min packing (quant.rs:316-327): lane t < 4 writes bytes
            // t, t+4, t+8 of the 12 from sub-blocks t and t+4
            {
                const int t = lane & 3;
                const int ls_a = __shfl_sync(0xffffffffu, lsq, t * 4), ls_b = __shfl_sync(0xffffffffu, lsq, t * 4 + 16);
                const int lm_a = __shfl_sync(0xffffffffu, lmq, t * 4), lm_b = __shfl_sync(0xffffffffu, lmq, t * 4 + 16);
                if (lane < 4) {
                    o[4 + t] = (uint8_t)(ls_a | ((ls_b >> 4) << 6));
                    o[8 + t] = (uint8_t)(lm_a | ((lm_b >> 4) << 6));
                    o[12 + t] = (uint8_t)((ls_b & 0xF) | ((lm_b & 0xF) << 4));
                }
            }
            if (lane == 0) {
                const uint16_t hd = f16_bits(d), hm = f16_bits(dmin);
                o[0] = (uint8_t)(hd & 0xFF);
                o[1] = (uint8_t)(hd >> 8);
                o[2] = (uint8_t)(hm & 0xFF);
                o[3] = (uint8_t)(hm >> 8);
            }
            __syncwarp();
            if (NMAX == 31) {
                uint8_t qh = 0;
#pragma unroll
                for (int chunk = 0; chunk < 4; chunk++) {
                    if (L[chunk * 64 + lane] >= 16) qh |= (uint8_t)(1u << (chunk * 2));
                    if (L[chunk * 64 + 32 + lane] >= 16) qh |= (uint8_t)(2u << (chunk * 2));
                }
                o[16 + lane] = qh;
#pragma unroll
                for (int t = 0; t < 4; t++) {
                    const int b = lane * 4 + t, chunk = b >> 5, l = b & 31;
                    o[48 + b] = (uint8_t)((L[chunk * 64 + l] & 0xF) | ((L[chunk * 64 + 32 + l] & 0xF) << 4));
                }
            } else {
#pragma unroll
                for (int t = 0; t < 4; t++) {
                    const int b = lane * 4 + t, chunk = b >> 5, l = b & 31;
                    o[16 + b] = (uint8_t)((L[chunk * 64 + l] & 0xF) | (L[chunk * 64 + 32 + l] << 4));
                }
            }
        }
        __syncwarp();
        if constexpr (!FUSE) store_block(a.dst + row * a.dst_row_bytes + sbi * BB, o, BB, !Q2 && a.dst_aligned16 != 0, lane);
        __syncwarp();
    };
    if constexpr (!FUSE) {
        for (int64_t g = (int64_t)blockIdx.x * kQkx3Warps + wid; g < total; g += nwarps) unit(g);
    } else {
        constexpr uint32_t TYPE = Q2 ? SHC_TYPE_Q2_K : NMAX == 31 ? SHC_TYPE_Q5_K : SHC_TYPE_Q4_K;
        FuseIter<NWE> it(a, nsb, wid);
        uint32_t fk = 0;
        while (it.next()) {
            if (it.valid) unit(it.row * nsb + it.unit);
            fuse_emit<TYPE, 0>(*F, wid, fk, it.valid, a, it.row, it.unit, W->out, lane);
        }
    }
}

template <int NMAX, bool FUSE>
__global__ void __launch_bounds__(FUSE ? 512 : 256, FUSE ? 1 : 2) enc_qk45_kernel(EncArgs a) {
    extern __shared__ __align__(16) uint8_t qkx3_smem[];
    qkx3_super_blocks<32, NMAX, FUSE>(a, qkx3_smem);
}

// Q2_K (ggml block_q2_K layout): make_qkx3_quants (quant.rs:77-141, nmax 3,
// rmin -0.9, rdelta 0.05, 37 grids) per 16-element sub-block, 4-bit scale and
// min codes against the super-block's largest scale and min, 2-bit levels.
template <bool FUSE>
__global__ void __launch_bounds__(256, 2) enc_q2_k_kernel(EncArgs a) {
    extern __shared__ __align__(16) uint8_t qkx3_smem[];
    qkx3_super_blocks<16, 3, FUSE>(a, qkx3_smem);
}

// ---------------------------------------------------------------------------
// Legacy 32-blocks (quant.rs:171-229): Q4_0/Q5_0 with make_qx_quants (nmax 8
// or 16), Q4_1/Q5_1 with make_qkx3_quants (nmax 15 or 31); these keep the
// search's level vector, so the winner's levels are recomputed from its
// grid.  A warp encodes 8 consecutive blocks (flat over the tensor's blocks,
// rows may change inside a group), 4 lanes per block.
// KIND: 0 Q4_0, 1 Q5_0, 2 Q4_1, 3 Q5_1
// ---------------------------------------------------------------------------
// Levels (l + nmax) that make_qx_quants (quant.rs:34-73) writes for one
// 32-element block of row `row` starting at column `col`, recomputed
// serially by one lane; false when the block accepts no grid and writes
// nothing.  Same arithmetic, in the same order, as the cooperative search
// in enc_legacy_kernel.
template <int NMAX>
__device__ bool legacy_sym_levels(const EncArgs &a, int64_t row, int64_t col, uint8_t *out) {
    constexpr float FN = (float)NMAX;
    float x[32], w[32];
    const float sig = a.sigma2[row];
    const float *imr = im_row(a.im, a.src.ne0, a.row0 + row * a.row_step);
    for (int m = 0; m < 4; m++) {
        float v[8], base[8];
        load8(a.src, row, col + m * 8, v);
        load_im8(imr, col + m * 8, base);
        for (int k = 0; k < 8; k++) {
            x[m * 8 + k] = v[k];
            w[m * 8 + k] = base[k] * sqrtf(sig + v[k] * v[k]);
        }
    }
    float amax = 0.0f, mx = 0.0f;
    for (int i = 0; i < 32; i++) {
        const float av = fabsf(x[i]);
        if (av > amax) { amax = av; mx = x[i]; }
    }
    if (amax < kGroupMaxEps) {
        for (int i = 0; i < 32; i++) out[i] = (uint8_t)NMAX;
        return true;
    }
    float best = 0.0f;
    bool first = true;
    int win = -1;
    for (int t = 0; t < 19; t++) {
        const float iscale = -(FN + 0.1f * (float)(t - 9)) / mx;
        float sumlx = 0.0f, suml2 = 0.0f;
        for (int i = 0; i < 32; i++) {
            const float l = round_clamp_f(iscale * x[i], -FN, FN - 1.0f);
            sumlx += w[i] * x[i] * l;
            suml2 += w[i] * (l * l);
        }
        if (suml2 > 0.0f && (first || sumlx * sumlx > best * suml2)) {
            best = (sumlx / suml2) * sumlx;
            first = false;
            win = t;
        }
    }
    if (win < 0) return false;
    const float iscale = -(FN + 0.1f * (float)(win - 9)) / mx;
    for (int i = 0; i < 32; i++) out[i] = (uint8_t)(clampi(nearest_int(iscale * x[i]), -NMAX, NMAX - 1) + NMAX);
    return true;
}

// FUSE: the fused error table (fuse.cuh): warps 0-6 encode a row's
// 256-element unit each, warp 7 folds.
template <int KIND, bool FUSE>
__global__ void __launch_bounds__(256) enc_legacy_kernel(EncArgs a) {
    constexpr bool SYM = KIND < 2;
    constexpr int NMAX = KIND == 0 ? 8 : KIND == 1 ? 16 : KIND == 2 ? 15 : 31;
    constexpr int BB = KIND == 0 ? 18 : KIND == 1 ? 22 : KIND == 2 ? 20 : 24;
    constexpr float FN = (float)NMAX;
    __shared__ float s_x[8][8 * 33];
    __shared__ float s_w[8][8 * 33];
    __shared__ float2 s_cand[8][8][20];
    __shared__ __align__(16) uint8_t s_out[8][8 * BB];
    __shared__ uint8_t s_l[8][256];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int b = lane >> 2, q = lane & 3;
    const int64_t ne0 = a.src.ne0, bpr = ne0 >> 5, nblk = a.n_rows * bpr;
    const int64_t ngrp = (nblk + 7) >> 3;
    constexpr int NWE = 7;
    extern __shared__ __align__(16) uint8_t legacy_fuse_smem[];
    FuseSmem<NWE> *F = reinterpret_cast<FuseSmem<NWE> *>(legacy_fuse_smem);
    const int64_t upr = (bpr + 7) >> 3;
    if constexpr (FUSE) {
        fuse_setup(*F);
        if (wid == NWE) {
            fuse_fold(*F, a, upr, lane);
            return;
        }
    }
    // blocks [blk0, blk0 + nb) of the tensor, 4 lanes per block
    auto unit = [&](int64_t blk0, int nb) {
        const int64_t blk = blk0 + b;
        const bool valid = b < nb;
        const int64_t row = valid ? blk / bpr : 0;
        const int64_t col = valid ? (blk - row * bpr) * 32 : 0;
        float v[8], base[8];
        float sig = 0.0f;
        if (valid) {
            load8(a.src, row, col + q * 8, v);
            load_im8(im_row(a.im, ne0, a.row0 + row * a.row_step), col + q * 8, base);
            sig = a.sigma2[row];
        } else {
#pragma unroll
            for (int k = 0; k < 8; k++) { v[k] = 0.0f; base[k] = 1.0f; }
        }
#pragma unroll
        for (int k = 0; k < 8; k++) {
            s_x[wid][b * 33 + q * 8 + k] = v[k];
            s_w[wid][b * 33 + q * 8 + k] = base[k] * sqrtf(sig + v[k] * v[k]);
        }
        __syncwarp();
        float x[32], w[32];
#pragma unroll
        for (int i = 0; i < 32; i++) {
            x[i] = s_x[wid][b * 33 + i];
            w[i] = s_w[wid][b * 33 + i];
        }
        float d_out = 0.0f, m_out = 0.0f, win_iscale = 0.0f, win_vmin = 0.0f;
        int mode = 0;  // SYM: 0 all nmax (tiny block), 1 levels from win_iscale
                       // ASYM: 0 all zero (degenerate), 1 levels from win_iscale over x - vmin
        if (SYM) {
            // make_qx_quants (quant.rs:34-73)
            float amax = 0.0f, mx = 0.0f;
#pragma unroll
            for (int i = 0; i < 32; i++) {
                const float av = fabsf(x[i]);
                if (av > amax) { amax = av; mx = x[i]; }
            }
            const bool live = !(amax < kGroupMaxEps);
            if (live) {
                for (int t = q; t < 19; t += 4) {
                    const float iscale = -(FN + 0.1f * (float)(t - 9)) / mx;
                    float sumlx = 0.0f, suml2 = 0.0f;
#pragma unroll
                    for (int i = 0; i < 32; i++) {
                        const float l = round_clamp_f(iscale * x[i], -FN, FN - 1.0f);
                        sumlx += w[i] * x[i] * l;
                        suml2 += w[i] * (l * l);
                    }
                    s_cand[wid][b][t] = make_float2(sumlx, suml2);
                }
            }
            __syncwarp();
            if (live) {
                float best = 0.0f, best_scale = 0.0f;
                bool first = true;
                int win = -1;
                for (int t = 0; t < 19; t++) {
                    const float2 c = s_cand[wid][b][t];
                    if (c.y > 0.0f && (first || c.x * c.x > best * c.y)) {
                        const float sc = c.x / c.y;
                        best_scale = sc;
                        best = sc * c.x;
                        first = false;
                        win = t;
                    }
                }
                d_out = best_scale;
                if (win >= 0) {
                    mode = 1;
                    win_iscale = -(FN + 0.1f * (float)(win - 9)) / mx;
                } else {
                    mode = 2;  // no grid accepted: the previous block's levels stay (below)
                }
            }
        } else {
            // make_qkx3_quants (quant.rs:77-141), rmin -0.9, rdelta 0.05, 36 steps
            float vmin = INFINITY, vmax = -INFINITY;
#pragma unroll
            for (int i = 0; i < 32; i++) vmin = rminf(vmin, x[i]);
            vmin = rminf(vmin, 0.0f);
#pragma unroll
            for (int i = 0; i < 32; i++) vmax = rmaxf(vmax, x[i]);
            const bool degen = vmax <= vmin;
            const float range = vmax - vmin;
            const float iscale0 = FN / range;
            const float scale0 = 1.0f / iscale0;
            float init_err = 0.0f, best_e = 0.0f, best_s = 0.0f, best_m = 0.0f;
            int best_j = -1;
            if (!degen) {
                float sum_w = 0.0f, sum_x = 0.0f;
#pragma unroll
                for (int i = 0; i < 32; i++) {
                    sum_w += w[i];
                    sum_x += w[i] * x[i];
                }
                for (int j = q; j < 38; j += 4) {
                    const float iscale = j == 37 ? iscale0 : (-0.9f + 0.05f * (float)j + FN) / range;
                    float sl = 0.0f, sl2 = 0.0f, sxl = 0.0f;
                    float l[32];
#pragma unroll
                    for (int i = 0; i < 32; i++) {
                        l[i] = round_clamp0_f(iscale * (x[i] - vmin), FN);
                        const float wl = w[i] * l[i];
                        sl += wl;
                        sl2 += w[i] * (l[i] * l[i]);
                        sxl += wl * x[i];
                    }
                    float ts, tm;
                    bool ok;
                    if (j == 37) {
                        ts = scale0;
                        tm = vmin;
                        ok = true;
                    } else {
                        const float D = sum_w * sl2 - sl * sl;
                        ok = D > 0.0f;
                        ts = (sum_w * sxl - sum_x * sl) / D;
                        tm = (sl2 * sum_x - sl * sxl) / D;
                        if (tm > 0.0f) {
                            tm = 0.0f;
                            ts = sl2 > 0.0f ? sxl / sl2 : 0.0f;
                        }
                    }
                    if (ok) {
                        float err = 0.0f;
#pragma unroll
                        for (int i = 0; i < 32; i++) {
                            const float diff = ts * l[i] + tm - x[i];
                            err += w[i] * diff * diff;
                        }
                        if (j == 37) {
                            init_err = err;
                        } else if (err == err && (best_j < 0 || err < best_e)) {
                            best_e = err;
                            best_j = j;
                            best_s = ts;
                            best_m = tm;
                        }
                    }
                }
            }
            __syncwarp();
#pragma unroll
            for (int off = 1; off <= 2; off <<= 1) {
                const float oe = __shfl_xor_sync(0xffffffffu, best_e, off);
                const int oj = __shfl_xor_sync(0xffffffffu, best_j, off);
                const float os = __shfl_xor_sync(0xffffffffu, best_s, off);
                const float om = __shfl_xor_sync(0xffffffffu, best_m, off);
                if (oj >= 0 && (best_j < 0 || oe < best_e || (oe == best_e && oj < best_j))) {
                    best_e = oe;
                    best_j = oj;
                    best_s = os;
                    best_m = om;
                }
            }
            init_err = __shfl_sync(0xffffffffu, init_err, (lane & ~3) | 1);
            if (degen) {
                d_out = 0.0f;
                m_out = vmin;
                mode = 0;
            } else if (best_j >= 0 && best_e < init_err) {
                d_out = best_s;
                m_out = best_m;
                mode = 1;
                win_iscale = (-0.9f + 0.05f * (float)best_j + FN) / range;
            } else {
                d_out = scale0;
                m_out = vmin;
                mode = 1;
                win_iscale = iscale0;
            }
            win_vmin = vmin;
        }
        // levels of this lane's 8 elements
        if (!SYM || mode != 2) {
#pragma unroll
            for (int k = 0; k < 8; k++) {
                int l;
                if (SYM) l = mode == 1 ? clampi(nearest_int(win_iscale * v[k]), -NMAX, NMAX - 1) + NMAX : NMAX;
                else l = mode == 1 ? clampi(nearest_int(win_iscale * (v[k] - win_vmin)), 0, NMAX) : 0;
                s_l[wid][lane * 8 + k] = (uint8_t)l;
            }
        } else if (q == 0) {
            // make_qx_quants wrote nothing: the reference's level buffer `ls`
            // outlives the block loop (quant.rs:172, 186) and still holds the
            // levels of the nearest earlier block of this row that wrote
            // some, or zeros (it starts zeroed for every row).  Rare (a block
            // whose weighted level energy is zero or NaN for every grid), so
            // one lane walks back through the row recomputing blocks.
            uint8_t *lv = &s_l[wid][b * 32];
            bool found = false;
            for (int64_t c = col - 32; c >= 0 && !found; c -= 32) found = legacy_sym_levels<NMAX>(a, row, c, lv);
            if (!found)
                for (int i = 0; i < 32; i++) lv[i] = 0;
        }
        __syncwarp();
        {
            uint8_t *o = s_out[wid] + b * BB;
            const uint8_t *L = s_l[wid] + b * 32;
            if (q == 0) {
                const uint16_t hd = f16_bits(d_out);
                o[0] = (uint8_t)(hd & 0xFF);
                o[1] = (uint8_t)(hd >> 8);
                if (!SYM) {
                    const uint16_t hm = f16_bits(m_out);
                    o[2] = (uint8_t)(hm & 0xFF);
                    o[3] = (uint8_t)(hm >> 8);
                }
                if (KIND == 1 || KIND == 3) {
                    uint32_t qh = 0;
                    for (int j = 0; j < 32; j++) qh |= ((uint32_t)((L[j] >> 4) & 1)) << j;
                    const int at = KIND == 1 ? 2 : 4;
                    o[at] = (uint8_t)qh;
                    o[at + 1] = (uint8_t)(qh >> 8);
                    o[at + 2] = (uint8_t)(qh >> 16);
                    o[at + 3] = (uint8_t)(qh >> 24);
                }
            }
            const int qs = KIND == 0 ? 2 : KIND == 1 ? 6 : KIND == 2 ? 4 : 8;
#pragma unroll
            for (int t = 0; t < 4; t++) {
                const int j = q * 4 + t;
                o[qs + j] = (KIND == 2 || KIND == 0) ? (uint8_t)((L[j] & 0xF) | (L[j + 16] << 4))
                                                     : (uint8_t)((L[j] & 0xF) | ((L[j + 16] & 0xF) << 4));
            }
        }
        __syncwarp();
        if constexpr (!FUSE) store_block(a.dst + blk0 * BB, s_out[wid], nb * BB, a.dst_aligned16 && nb == 8, lane);
        __syncwarp();
    };
    if constexpr (!FUSE) {
        for (int64_t g = (int64_t)blockIdx.x * 8 + wid; g < ngrp; g += (int64_t)gridDim.x * 8) {
            const int64_t blk0 = g * 8;
            unit(blk0, (int)(nblk - blk0 < 8 ? nblk - blk0 : 8));
        }
    } else {
        constexpr uint32_t TYPE = KIND == 0 ? SHC_TYPE_Q4_0 : KIND == 1 ? SHC_TYPE_Q5_0 : KIND == 2 ? SHC_TYPE_Q4_1
                                                                                                 : SHC_TYPE_Q5_1;
        FuseIter<NWE> it(a, upr, wid);
        uint32_t fk = 0;
        while (it.next()) {
            const int64_t left = bpr - it.unit * 8;
            if (it.valid) unit(it.row * bpr + it.unit * 8, (int)(left < 8 ? left : 8));
            fuse_emit<TYPE, BB>(*F, wid, fk, it.valid, a, it.row, it.unit, s_out[wid], lane);
        }
    }
}

// ---------------------------------------------------------------------------
// Elementwise encodings (quant.rs:546-560): F32 copy, F16 round-to-nearest-
// even, BF16 by truncating the low 16 bits (`(v.to_bits() >> 16) as u16`).
// ---------------------------------------------------------------------------
__global__ void enc_plain_kernel(uint32_t type, EncArgs a) {
    const int64_t ne0 = a.src.ne0, n = a.n_rows * ne0;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = e / ne0, col = e - row * ne0;
        const float x = load1(a.src, row, col);
        if (type == SHC_TYPE_F32) {
            reinterpret_cast<float *>(a.dst)[e] = x;
        } else {
            const uint16_t h = type == SHC_TYPE_F16 ? f16_bits(x) : (uint16_t)(__float_as_uint(x) >> 16);
            reinterpret_cast<uint16_t *>(a.dst)[e] = h;
        }
    }
}

// Error table of an elementwise candidate (F32, F16, BF16): the fused
// layout of fuse.cuh with the round trip in place of an encoder; 7 warps
// compute terms, warp 7 folds.
template <uint32_t TYPE>
__global__ void __launch_bounds__(256) plain_fused_kernel(EncArgs a) {
    constexpr int NWE = 7;
    extern __shared__ __align__(16) uint8_t plain_fuse_smem[];
    FuseSmem<NWE> *F = reinterpret_cast<FuseSmem<NWE> *>(plain_fuse_smem);
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int64_t upr = (a.src.ne0 + 255) / 256;
    fuse_setup(*F);
    if (wid == NWE) {
        fuse_fold(*F, a, upr, lane);
        return;
    }
    FuseIter<NWE> it(a, upr, wid);
    uint32_t fk = 0;
    while (it.next()) fuse_emit_plain<TYPE>(*F, wid, fk, it.valid, a, it.row, it.unit, lane);
}

cudaError_t launch_plain(uint32_t type, const EncArgs &a, int num_sms, cudaStream_t st) {
    const int64_t n = a.n_rows * a.src.ne0;
    int64_t blocks = (n + 255) / 256;
    if (blocks > (int64_t)num_sms * 16) blocks = (int64_t)num_sms * 16;
    if (blocks < 1) blocks = 1;
    enc_plain_kernel<<<(unsigned)blocks, 256, 0, st>>>(type, a);
    return cudaGetLastError();
}

cudaError_t resident_blocks(const void *fn, int threads, size_t smem, int *per_sm) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    using Key = std::tuple<int, const void *, int, size_t>;
    static std::mutex mu;
    static std::map<Key, int> cache;
    const Key key{dev, fn, threads, smem};
    {
        std::lock_guard<std::mutex> lk(mu);
        auto it = cache.find(key);
        if (it != cache.end()) {
            *per_sm = it->second;
            return cudaSuccess;
        }
    }
    if (smem > 0) {
        e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    int n = 1;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, threads, smem);
    if (e != cudaSuccess) return e;
    if (n < 1) n = 1;
    std::lock_guard<std::mutex> lk(mu);
    cache[key] = n;
    *per_sm = n;
    return cudaSuccess;
}

// Grid for the persistent warp-per-super-block kernels: enough CTAs to fill
// every SM at the occupancy the kernel reaches, never more than the work.
static unsigned persistent_grid(const void *fn, int threads, int num_sms, int64_t work_warps) {
    int per_sm = 1;
    if (resident_blocks(fn, threads, 0, &per_sm) != cudaSuccess) per_sm = 1;
    int64_t want = (work_warps + threads / 32 - 1) / (threads / 32);
    int64_t cap = (int64_t)num_sms * per_sm;
    if (want > cap) want = cap;
    if (want < 1) want = 1;
    return (unsigned)want;
}

// Warp-per-super-block make_qkx3_quants kernels: dynamic shared memory of
// kQkx3Warps per-warp workspaces, a persistent grid of resident blocks.
template <int N>
static cudaError_t launch_qkx3(void (*fn)(EncArgs), const EncArgs &a, int num_sms, cudaStream_t st) {
    const size_t smem = kQkx3Warps * sizeof(Qkx3Warp<N>);
    int per_sm = 1;
    cudaError_t e = resident_blocks((const void *)fn, kQkx3Warps * 32, smem, &per_sm);
    if (e != cudaSuccess) return e;
    int64_t grid = (a.n_rows * (a.src.ne0 / 256) + kQkx3Warps - 1) / kQkx3Warps;
    const int64_t cap = (int64_t)num_sms * per_sm;
    if (grid > cap) grid = cap;
    if (grid < 1) grid = 1;
    fn<<<(unsigned)grid, kQkx3Warps * 32, smem, st>>>(a);
    return cudaGetLastError();
}

static cudaError_t launch_qx16(void (*fn)(EncArgs), const EncArgs &a, int num_sms, cudaStream_t st) {
    const size_t smem = 8 * sizeof(Qx16Warp);
    int per_sm = 1;
    cudaError_t e = resident_blocks((const void *)fn, 256, smem, &per_sm);
    if (e != cudaSuccess) return e;
    int64_t grid = (a.n_rows * (a.src.ne0 / 256) + 7) / 8;
    const int64_t cap = (int64_t)num_sms * per_sm;
    if (grid > cap) grid = cap;
    if (grid < 1) grid = 1;
    fn<<<(unsigned)grid, 256, smem, st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_kquant(uint32_t type, const EncArgs &a, int num_sms, cudaStream_t st) {
    switch (type) {
    case SHC_TYPE_Q8_0: {
        unsigned grid = persistent_grid((const void *)enc_q8_0_kernel<false>, 256, num_sms,
                                        (a.n_rows * (a.src.ne0 / 32) + 31) / 32);
        enc_q8_0_kernel<false><<<grid, 256, 0, st>>>(a);
        break;
    }
    case SHC_TYPE_Q6_K: return launch_qx16(enc_qx16_kernel<32, false>, a, num_sms, st);
    case SHC_TYPE_Q3_K: return launch_qx16(enc_qx16_kernel<4, false>, a, num_sms, st);
    case SHC_TYPE_Q2_K: return launch_qkx3<16>(enc_q2_k_kernel<false>, a, num_sms, st);
    case SHC_TYPE_Q4_K: return launch_qkx3<32>(enc_qk45_kernel<15, false>, a, num_sms, st);
    case SHC_TYPE_Q5_K: return launch_qkx3<32>(enc_qk45_kernel<31, false>, a, num_sms, st);
    case SHC_TYPE_Q4_0: case SHC_TYPE_Q5_0: case SHC_TYPE_Q4_1: case SHC_TYPE_Q5_1: {
        const int64_t ngrp = (a.n_rows * (a.src.ne0 / 32) + 7) / 8;
        const void *fn = type == SHC_TYPE_Q4_0 ? (const void *)enc_legacy_kernel<0, false>
                         : type == SHC_TYPE_Q5_0 ? (const void *)enc_legacy_kernel<1, false>
                         : type == SHC_TYPE_Q4_1 ? (const void *)enc_legacy_kernel<2, false>
                                                 : (const void *)enc_legacy_kernel<3, false>;
        unsigned grid = persistent_grid(fn, 256, num_sms, ngrp);
        if (type == SHC_TYPE_Q4_0) enc_legacy_kernel<0, false><<<grid, 256, 0, st>>>(a);
        else if (type == SHC_TYPE_Q5_0) enc_legacy_kernel<1, false><<<grid, 256, 0, st>>>(a);
        else if (type == SHC_TYPE_Q4_1) enc_legacy_kernel<2, false><<<grid, 256, 0, st>>>(a);
        else enc_legacy_kernel<3, false><<<grid, 256, 0, st>>>(a);
        break;
    }
    default:
        return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

// Fused launch: NWE encoder warps + the fold warp per CTA, dynamic shared
// memory = the encoders' workspaces (ws_bytes) + the fold slots, groups of
// rows sized for the resident CTAs, one CTA per group up to the resident
// count.
template <int NWE>
static cudaError_t launch_fused(void (*fn)(EncArgs), EncArgs a, size_t ws_bytes, int64_t upr, int num_sms,
                                cudaStream_t st) {
    const size_t smem = ws_bytes + sizeof(FuseSmem<NWE>);
    constexpr int threads = (NWE + 1) * 32;
    int per_sm = 1;
    cudaError_t e = resident_blocks((const void *)fn, threads, smem, &per_sm);
    if (e != cudaSuccess) return e;
    const int64_t cap = (int64_t)num_sms * per_sm;
    a.fuse_rows = fuse_rows_per_group(a.n_rows, upr, NWE, cap);
    int64_t grid = (a.n_rows + a.fuse_rows - 1) / a.fuse_rows;
    if (grid > cap) grid = cap;
    if (grid < 1) grid = 1;
    fn<<<(unsigned)grid, threads, smem, st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_kquant_fused(uint32_t type, const EncArgs &a, int num_sms, cudaStream_t st) {
    if (!a.err || a.n_rows < 1) return cudaErrorInvalidValue;
    const int64_t ne0 = a.src.ne0, upr = (ne0 + 255) / 256;
    switch (type) {
    case SHC_TYPE_Q8_0: return launch_fused<7>(enc_q8_0_kernel<true>, a, 0, upr, num_sms, st);
    case SHC_TYPE_Q6_K:
        return launch_fused<15>(enc_qx16_kernel<32, true>, a, 15 * sizeof(Qx16Warp), upr, num_sms, st);
    case SHC_TYPE_Q3_K:
        return launch_fused<15>(enc_qx16_kernel<4, true>, a, 15 * sizeof(Qx16Warp), upr, num_sms, st);
    case SHC_TYPE_Q2_K:
        return launch_fused<7>(enc_q2_k_kernel<true>, a, 7 * sizeof(Qkx3Warp<16>), upr, num_sms, st);
    case SHC_TYPE_Q4_K:
        return launch_fused<15>(enc_qk45_kernel<15, true>, a, 15 * sizeof(Qkx3Warp<32>), upr, num_sms, st);
    case SHC_TYPE_Q5_K:
        return launch_fused<15>(enc_qk45_kernel<31, true>, a, 15 * sizeof(Qkx3Warp<32>), upr, num_sms, st);
    case SHC_TYPE_Q4_0: return launch_fused<7>(enc_legacy_kernel<0, true>, a, 0, upr, num_sms, st);
    case SHC_TYPE_Q5_0: return launch_fused<7>(enc_legacy_kernel<1, true>, a, 0, upr, num_sms, st);
    case SHC_TYPE_Q4_1: return launch_fused<7>(enc_legacy_kernel<2, true>, a, 0, upr, num_sms, st);
    case SHC_TYPE_Q5_1: return launch_fused<7>(enc_legacy_kernel<3, true>, a, 0, upr, num_sms, st);
    case SHC_TYPE_F32: return launch_fused<7>(plain_fused_kernel<SHC_TYPE_F32>, a, 0, upr, num_sms, st);
    case SHC_TYPE_F16: return launch_fused<7>(plain_fused_kernel<SHC_TYPE_F16>, a, 0, upr, num_sms, st);
    case SHC_TYPE_BF16: return launch_fused<7>(plain_fused_kernel<SHC_TYPE_BF16>, a, 0, upr, num_sms, st);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace shc
