/* shoehorn_cuda.h — C ABI of the B200 (sm_100a) quantization library.
 *
 * Drop-in boundary for shoehorn's quantization hot path.  The reference has no
 * FFI layer; its replaceable seam is the Rust row API in src/quant.rs:
 *
 *   pub fn encode_row(ty: GgmlType, x: &[f32], im: Option<&[f32]>, out: &mut Vec<u8>)   quant.rs:543
 *   pub fn decode_row(ty: GgmlType, data: &[u8], n: usize, out: &mut Vec<f32>)        quant.rs:581
 *   pub fn row_error(ty: GgmlType, x: &[f32], im: Option<&[f32]>) -> f64             quant.rs:618
 *
 * called once per row from rayon workers in the error-table loop
 * (main.rs:549-563) and in encode_tensor (main.rs:663-686).  Per-row calls
 * across an FFI would serialise the GPU, so the entry points here are
 * tensor-granular: one call covers a contiguous range of rows of one tensor
 * and produces exactly the bytes / errors the per-row loop would.
 *
 * Conventions
 *   - Every function returns an int status (SHC_OK == 0, negative on error);
 *     nothing throws across the ABI and no kernel traps.
 *   - Pointers are caller-owned.  "Device" entry points take device pointers
 *     and are asynchronous on the given CUDA stream (NULL = legacy default
 *     stream); completion and the device status word are collected by
 *     shc_sync().  "Host" entry points take host pointers (pinned or pageable)
 *     and return when the result is in host memory.
 *   - Rows are contiguous: row r of a tensor starts at element r * ne0.
 *   - The imatrix follows imatrix.rs:124-141 row_slice: length ne0 applies to
 *     every row; a multiple k*ne0 selects matrix (row0 + r) / rows_per_mat,
 *     clamped to k-1; any other length (or NULL) means "no imatrix", which
 *     selects each type's unweighted fallback exactly as the reference does.
 *   - A context is bound to one device.  Calls on one context may come from
 *     several host threads; work is stream-ordered and per-call temporaries
 *     are stream-ordered allocations, so calls on different streams do not
 *     share scratch.
 */
#ifndef SHOEHORN_CUDA_H
#define SHOEHORN_CUDA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids, as in the reference's GgmlType (gguf.rs:36-83). */
#define SHC_TYPE_F32 0u
#define SHC_TYPE_F16 1u
#define SHC_TYPE_Q4_0 2u
#define SHC_TYPE_Q4_1 3u
#define SHC_TYPE_Q5_0 6u
#define SHC_TYPE_Q5_1 7u
#define SHC_TYPE_Q8_0 8u
/* Q2_K and Q3_K have no encoder in the reference (its GgmlType stops at the
 * types above); blocks follow ggml's block_q2_K (84 bytes) and block_q3_K
 * (110 bytes) layouts with the reference's K-quant search routines. */
#define SHC_TYPE_Q2_K 10u
#define SHC_TYPE_Q3_K 11u
#define SHC_TYPE_Q4_K 12u
#define SHC_TYPE_Q5_K 13u
#define SHC_TYPE_Q6_K 14u
#define SHC_TYPE_IQ2_XXS 16u
#define SHC_TYPE_IQ2_XS 17u
#define SHC_TYPE_IQ3_XXS 18u
#define SHC_TYPE_IQ4_NL 20u
#define SHC_TYPE_IQ3_S 21u
#define SHC_TYPE_IQ2_S 22u
#define SHC_TYPE_IQ4_XS 23u
#define SHC_TYPE_BF16 30u

/* Source element types of the rows (the reference decodes F32/F16/BF16
 * storage to f32 before encoding, quant.rs:581-597). */
#define SHC_SRC_F32 0u
#define SHC_SRC_F16 1u
#define SHC_SRC_BF16 30u

/* Status codes. */
#define SHC_OK 0
#define SHC_EINVAL -1        /* unknown type, bad sizes, misaligned pointer */
#define SHC_ECUDA -2         /* a CUDA runtime call failed */
#define SHC_EOFFGRID -3      /* an IQ point ended off the lattice (quant_iq.rs:386,538,705,890 assert) */
#define SHC_ENONEIGHBOUR -4  /* IQ neighbour search found no finite candidate (quant_iq.rs:162 would panic) */
#define SHC_ETIMEOUT -5      /* bounded wait expired; the work may still be running */
#define SHC_ENOMEM -6        /* device or pinned host allocation failed */
#define SHC_ENODEV -7        /* no usable CUDA device / not an sm_100 device */

typedef struct shc_ctx shc_ctx;

/* Context bound to one CUDA device.  Builds the IQ lattice maps and neighbour
 * lists on the host exactly as quant_iq.rs:44-133 (build_grid/expand_kgrid)
 * and uploads them with the decode grids, once.  Replaces the OnceLock grids
 * of quant_iq.rs:114-133. */
int shc_init(int device, shc_ctx **out);
int shc_free(shc_ctx *ctx);
const char *shc_status_string(int status);

/* gguf.rs:109-113 GgmlType::row_bytes; -1 if the type is unknown or ne0 is
 * not a multiple of its block size. */
int64_t shc_row_bytes(uint32_t ggml_type, int64_t ne0);
/* 1 if shc_encode_rows supports ggml_type, else 0. */
int shc_type_supported(uint32_t ggml_type);

/* Encode n_rows rows of length ne0 into ggml_type (device pointers).
 * Replaces the per-row loop of encode_tensor (main.rs:672-683) over
 * quant.rs:543 encode_row.  dst receives n_rows * shc_row_bytes(type, ne0)
 * bytes, row-major, bit-identical to encode_row on each row.  row0 is the
 * global index of the first row (for the imatrix matrix selection). */
int shc_encode_rows(shc_ctx *ctx, uint32_t ggml_type, uint32_t src_type, const void *src, int64_t n_rows,
                    int64_t ne0, const float *imatrix, int64_t imatrix_len, int64_t rows_per_mat, int64_t row0,
                    uint8_t *dst, void *stream);

/* Decode n_rows encoded rows to f32 (device pointers); quant.rs:581 decode_row. */
int shc_decode_rows(shc_ctx *ctx, uint32_t ggml_type, const uint8_t *src, int64_t n_rows, int64_t ne0, float *dst,
                    void *stream);

/* Fused quantize -> dequantize -> weighted squared error for the sampled rows
 * r = 0, row_step, 2*row_step, ... < n_rows, for each of n_types candidate
 * types (device pointers).  err[t * n_sampled + i] receives
 * quant.rs:618 row_error(types[t], row(i*row_step), im) as the reference
 * computes it (f64 sum in element order); n_sampled = ceil(n_rows/row_step).
 * One kernel launch per block-quantized candidate encodes, decodes and folds
 * the error with the codes held in shared memory (plus one row sigma^2 pass
 * shared by the K-quant candidates); a NaN error is stored as the default
 * quiet NaN.  The caller sums rows in row order and scales by
 * n_rows / n_sampled (main.rs:546-560). */
int shc_row_errors(shc_ctx *ctx, const uint32_t *types, int n_types, uint32_t src_type, const void *src,
                   int64_t n_rows, int64_t ne0, const float *imatrix, int64_t imatrix_len, int64_t rows_per_mat,
                   int64_t row0, int64_t row_step, double *err, void *stream);

/* Wait for all work queued on stream (bounded by timeout_ms; <0 = no bound)
 * and return the first device-side status raised by any kernel of this
 * context since the previous shc_sync (the status word is then cleared). */
int shc_sync(shc_ctx *ctx, void *stream, int64_t timeout_ms);

/* Host-buffer entry point: the end-to-end call a host program makes.
 * host_src holds n_rows*ne0 elements of src_type, host_dst receives
 * n_rows*row_bytes bytes.  Rows stream through the device in chunks with
 * host->device copies, encoding and device->host copies overlapped on
 * separate streams.  Pinned (page-locked) host buffers are copied directly;
 * pageable ones are staged through the context's pinned buffers. */
int shc_encode_tensor_host(shc_ctx *ctx, uint32_t ggml_type, uint32_t src_type, const void *host_src,
                           int64_t n_rows, int64_t ne0, const float *host_imatrix, int64_t imatrix_len,
                           int64_t rows_per_mat, int64_t row0, uint8_t *host_dst, int64_t timeout_ms);

/* Host-buffer fused error table (see shc_row_errors); err is a host array
 * of n_types * n_sampled doubles. */
int shc_row_errors_host(shc_ctx *ctx, const uint32_t *types, int n_types, uint32_t src_type, const void *host_src,
                        int64_t n_rows, int64_t ne0, const float *host_imatrix, int64_t imatrix_len,
                        int64_t rows_per_mat, int64_t row0, int64_t row_step, double *err, int64_t timeout_ms);

/* Allocation-free encode for Q4_K, Q5_K and Q6_K.  No counterpart in the
 * reference (its CPU encoders allocate freely).
 *
 * shc_encode_rows draws its per-row sigma^2 scratch from CUDA's
 * stream-ordered allocator.  Some callers cannot allocate device memory at
 * the point where they encode: a host program whose own allocator reserved
 * the GPU's memory up front (a cudaMalloc from the library would then fail
 * or fragment that pool), or one that must not risk the device-wide
 * synchronisation cudaMalloc/cudaFree can cause in the middle of its work.
 * This entry point makes no allocation at all; its scratch is a fixed buffer
 * of SHC_NOALLOC_MAX_ROWS floats (256 KiB) compiled into the library, held
 * on every GPU that loads the library until the process exits.
 *
 *  - Runs on the calling thread's current CUDA device, asynchronously on
 *    `stream`; src, imatrix and dst are caller-owned device pointers with the
 *    same meaning and the same output bytes as shc_encode_rows.
 *  - The first call on each device looks up the buffer's device address;
 *    make that first call before any stream capture on that device.
 *  - n_rows > SHC_NOALLOC_MAX_ROWS returns SHC_ETOOLARGE and launches
 *    nothing; split larger tensors into row ranges (row0 keeps the imatrix
 *    selection right).
 *  - One buffer is shared by every call on a device and keeps the last
 *    call's contents.  Each call writes every entry it reads before reading
 *    it, so nothing needs clearing; but calls whose work overlaps on the GPU
 *    (different streams or host threads) race on it: issue them on one
 *    stream. */
#define SHC_ETOOLARGE -8
#define SHC_NOALLOC_MAX_ROWS 65536
int shc_encode_rows_noalloc(uint32_t ggml_type, uint32_t src_type, const void *src, int64_t n_rows, int64_t ne0,
                            const float *imatrix, int64_t imatrix_len, int64_t rows_per_mat, int64_t row0,
                            uint8_t *dst, void *stream);

/* Number of kernel launches issued by this context so far (instrumentation
 * for benchmarks). */
int64_t shc_launch_count(const shc_ctx *ctx);

/* Host-only introspection of the IQ lattice structures the encoders search
 * (replaces the public grid_iq2xxs()/grid_iq2xs()/grid_iq2s()/grid_iq3xxs()/
 * grid_iq3s() accessors, quant_iq.rs:114-133).  which: 0 IQ2_XXS, 1 IQ2_XS,
 * 2 IQ2_S, 3 IQ3_XXS, 4 IQ3_S.  The map is compacted to the lattice indices
 * the encoders can produce: IQ2 index sum(l_k * 3^k), l_k in 0..2 (6561
 * entries); IQ3 index sum(l_k << 3k), l_k in 0..7 (4096 entries).  Entries
 * >= 0 are grid indices; < 0 are -(offset+1) into `neighbours`, where
 * neighbours[offset] is a count followed by that many entries
 * (grid index | packed lattice coordinates << 16), ordered exactly as the
 * reference's neighbour lists.  Pass NULL outputs to query the sizes.
 * Needs no GPU. */
int shc_grid_info(int which, int32_t *grid_size, int32_t *map_size, int64_t *n_neighbours, int32_t *map_out,
                  uint32_t *neighbours_out);

#ifdef __cplusplus
}
#endif

#endif /* SHOEHORN_CUDA_H */
