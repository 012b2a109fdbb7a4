/* CPU oracle for the shoehorn quantization hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a strict-IEEE C restatement of the
 * reference's CPU encoders (src/quant.rs, src/quant_iq.rs) used to check the
 * CUDA library bit for bit and to time the reference algorithm on host cores.
 * Nothing in the shipped library links, loads or calls it.
 *
 * Build flags matter: -O2 -ffp-contract=off -fno-fast-math (no FMA
 * contraction, IEEE division/sqrt, gradual underflow), the same f32
 * semantics the reference gets from Rust.
 */
#pragma once
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes (shared meaning with the CUDA library). */
#define OQ_OK 0
#define OQ_EINVAL -1       /* unknown type, bad sizes */
#define OQ_EOFFGRID -3     /* an IQ point ended off the lattice (reference asserts) */
#define OQ_ENONEIGHBOUR -4 /* neighbour search found no finite candidate */

int64_t oq_row_bytes(uint32_t type, int64_t n);

/* quant.rs:543 encode_row: x[n] -> out[row_bytes(n)], im nullable (len n). */
int oq_encode_row(uint32_t type, const float *x, int64_t n, const float *im, uint8_t *out);
/* quant.rs:581 decode_row */
int oq_decode_row(uint32_t type, const uint8_t *data, int64_t n, float *out);
/* quant.rs:618 row_error: weighted squared error of encode+decode, f64. */
int oq_row_error(uint32_t type, const float *x, int64_t n, const float *im, double *err);

/* main.rs:663 encode_tensor for a BF16 source: rows decoded bits<<16, imatrix
 * sliced per imatrix.rs:124 row_slice, rows encoded in parallel chunks. */
int oq_encode_tensor_bf16(uint32_t type, const uint16_t *src, int64_t n_rows, int64_t ne0,
                          const float *im, int64_t im_len, int64_t rows_per_mat, uint8_t *dst,
                          int n_threads);
/* main.rs:549-563 measuring closure: per sampled row (r = 0, step, ...) the
 * row_error, written to err[i] for the i-th sampled row. */
int oq_row_errors_bf16(uint32_t type, const uint16_t *src, int64_t n_rows, int64_t ne0,
                       const float *im, int64_t im_len, int64_t rows_per_mat, int64_t row_step,
                       double *err, int n_threads);

/* IQ lattice structures (quant_iq.rs:44-133). which: 0 IQ2_XXS, 1 IQ2_XS,
 * 2 IQ2_S, 3 IQ3_XXS, 4 IQ3_S.  Copies out the kmap (kmap_size entries) and
 * the neighbour array; pass NULL to query sizes. */
int oq_grid_info(int which, int32_t *grid_size, int32_t *kmap_size, int64_t *n_neighbours,
                 int32_t *kmap_out, uint16_t *neighbours_out);

/* Helpers exposed for unit tests of the FP semantics. */
uint16_t oq_f32_to_f16(float x);
float oq_f16_to_f32(uint16_t h);
int32_t oq_nearest_int(float x);

#ifdef __cplusplus
}
#endif
