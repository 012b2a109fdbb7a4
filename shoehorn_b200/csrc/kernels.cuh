// Internal launch interface between the C ABI (api.cu) and the kernels.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace shc {

// Arguments shared by every encoder kernel.  Rows are addressed as
// i = 0..n_rows-1 in the source view (src.row_stride elements apart); the
// global row index used for the imatrix slice is row0 + i * row_step.
struct EncArgs {
    RowSrc src;
    ImSrc im;
    int64_t n_rows;
    int64_t row0;
    int64_t row_step;
    const float *sigma2;  // per-row sigma^2 (quant.rs:153), only for types that use it
    uint8_t *dst;         // n_rows * dst_row_bytes, rows contiguous
    int64_t dst_row_bytes;
    int *status;
    int dst_aligned16;
    // Fused error table (the *_fused launchers): err[i] receives row i's
    // weighted squared error; rows are handed out in groups of fuse_rows.
    double *err;
    int64_t fuse_rows;
};

// IQ lattice tables resident on the device (built on the host as
// quant_iq.rs:44-133 does, compacted to the lattice points the encoders can
// reach).  One entry per IQ2 grid variant (0 IQ2_XXS, 1 IQ2_XS, 2 IQ2_S) and
// IQ3 variant (3 IQ3_XXS, 4 IQ3_S).
struct IqTables {
    const int32_t *kmap[5];        // compact kmap: >=0 grid index, <0 -(offset+1) into neighbours
    const uint32_t *neighbours[5]; // [count, entry...]; entry = grid index | packed coords << 16
    const uint32_t *grid_coords[5];// per grid point: packed lattice coordinates (2 or 3 bits each)
    // Device copy of the lists in the layout the encoders scan: each list's
    // entries (IQ2_XXS 8-bit grid indices, the others 16-bit packed
    // coordinates) start on a four-entry boundary, padded to a multiple of
    // four with copies of the last entry; dkmap's off-grid entries hold
    // -(1 + first entry + (count << 19)).
    const int32_t *dkmap[5];  // kmap with offsets into `lists`
    const void *lists[5];
    int lists_bytes[5];
};

// Per-type constants (gguf.rs:86-107 block_layout).
__host__ __device__ inline int64_t block_elems(uint32_t t) {
    switch (t) {
    case SHC_TYPE_F32: case SHC_TYPE_F16: case SHC_TYPE_BF16: return 1;
    case SHC_TYPE_Q4_0: case SHC_TYPE_Q4_1: case SHC_TYPE_Q5_0: case SHC_TYPE_Q5_1: case SHC_TYPE_Q8_0:
    case SHC_TYPE_IQ4_NL: return 32;
    case SHC_TYPE_Q2_K: case SHC_TYPE_Q3_K: case SHC_TYPE_Q4_K: case SHC_TYPE_Q5_K: case SHC_TYPE_Q6_K:
    case SHC_TYPE_IQ2_XXS: case SHC_TYPE_IQ2_XS: case SHC_TYPE_IQ2_S: case SHC_TYPE_IQ3_XXS: case SHC_TYPE_IQ3_S:
    case SHC_TYPE_IQ4_XS: return 256;
    default: return 0;
    }
}
__host__ __device__ inline int64_t block_bytes(uint32_t t) {
    switch (t) {
    case SHC_TYPE_F32: return 4;
    case SHC_TYPE_F16: case SHC_TYPE_BF16: return 2;
    case SHC_TYPE_Q4_0: return 18;
    case SHC_TYPE_Q4_1: return 20;
    case SHC_TYPE_Q5_0: return 22;
    case SHC_TYPE_Q5_1: return 24;
    case SHC_TYPE_Q8_0: return 34;
    case SHC_TYPE_Q2_K: return 84;
    case SHC_TYPE_Q3_K: return 110;
    case SHC_TYPE_Q4_K: return 144;
    case SHC_TYPE_Q5_K: return 176;
    case SHC_TYPE_Q6_K: return 210;
    case SHC_TYPE_IQ2_XXS: return 66;
    case SHC_TYPE_IQ2_XS: return 74;
    case SHC_TYPE_IQ2_S: return 82;
    case SHC_TYPE_IQ3_XXS: return 98;
    case SHC_TYPE_IQ3_S: return 110;
    case SHC_TYPE_IQ4_NL: return 18;
    case SHC_TYPE_IQ4_XS: return 136;
    default: return 0;
    }
}
// Types whose encoder reads the row sigma^2 of quant.rs:544 (the IQ encoders
// recompute their own per super-block).
__host__ __device__ inline bool needs_sigma2(uint32_t t) {
    switch (t) {
    case SHC_TYPE_Q4_0: case SHC_TYPE_Q4_1: case SHC_TYPE_Q5_0: case SHC_TYPE_Q5_1: case SHC_TYPE_Q2_K:
    case SHC_TYPE_Q3_K: case SHC_TYPE_Q4_K: case SHC_TYPE_Q5_K: case SHC_TYPE_Q6_K: return true;
    default: return false;
    }
}
__host__ __device__ inline bool is_iq(uint32_t t) {
    switch (t) {
    case SHC_TYPE_IQ2_XXS: case SHC_TYPE_IQ2_XS: case SHC_TYPE_IQ2_S: case SHC_TYPE_IQ3_XXS: case SHC_TYPE_IQ3_S:
    case SHC_TYPE_IQ4_NL: case SHC_TYPE_IQ4_XS: return true;
    default: return false;
    }
}

// Resident blocks per SM of kernel `fn` launched with `threads` threads and
// `smem` bytes of dynamic shared memory on the current device, after raising
// the kernel's dynamic shared-memory limit to `smem`.  Computed once per
// (device, kernel, shape) and cached, so a launch pays no occupancy query.
cudaError_t resident_blocks(const void *fn, int threads, size_t smem, int *per_sm);

// Launchers (return a cudaError_t).  num_sms sizes the persistent grids.
cudaError_t launch_row_sigma2(const RowSrc &src, int64_t n_rows, float *out, cudaStream_t st);
cudaError_t launch_kquant(uint32_t type, const EncArgs &a, int num_sms, cudaStream_t st);
cudaError_t launch_plain(uint32_t type, const EncArgs &a, int num_sms, cudaStream_t st);
bool iq_supported(uint32_t type);
cudaError_t launch_iq(uint32_t type, const EncArgs &a, const IqTables &iq, int num_sms, cudaStream_t st);
cudaError_t launch_decode(uint32_t type, const uint8_t *src, int64_t n_rows, int64_t ne0, float *dst, int num_sms,
                          cudaStream_t st);
// Fused quantize -> dequantize -> weighted SSE of one candidate type: one
// launch, a.err[i] for every row i of the view, no codes written (a.dst
// unused).  The K-quant types read a.sigma2 like the plain encoders;
// launch_kquant_fused also takes the elementwise types (F32, F16, BF16).
cudaError_t launch_kquant_fused(uint32_t type, const EncArgs &a, int num_sms, cudaStream_t st);
cudaError_t launch_iq_fused(uint32_t type, const EncArgs &a, const IqTables &iq, int num_sms, cudaStream_t st);

}  // namespace shc
