// Counting build of the CPU oracle — TEST INFRASTRUCTURE (see opcount.hpp).
// Exports one entry point that encodes rows like oq_encode_row and reports
// the operations executed.
#include "opcount.hpp"

#include "../shoehorn_oracle.c"

#undef float

thread_local shoc::Counts shoc::counts;

extern "C" {
// Encodes n_rows f32 rows of ne0 (imatrix: ne0 floats or NULL) into dst and
// writes the executed-operation counts into out[6] (arith, cmp, sqrt, round,
// minmax, f64).  Returns the oracle's status.
int oc_encode_rows(uint32_t type, const float *x, int64_t n_rows, int64_t ne0, const float *im, uint8_t *dst,
                   uint64_t *out) {
    shoc::counts = {};
    int64_t rb = oq_row_bytes(type, ne0);
    if (rb < 0) return OQ_EINVAL;
    for (int64_t r = 0; r < n_rows; r++) {
        int rc = oq_encode_row(type, reinterpret_cast<const sh_cf *>(x + r * ne0), ne0,
                               reinterpret_cast<const sh_cf *>(im), dst + r * rb);
        if (rc != OQ_OK) return rc;
    }
    const shoc::Counts &c = shoc::counts;
    out[0] = c.arith; out[1] = c.cmp; out[2] = c.sqrt; out[3] = c.round; out[4] = c.minmax; out[5] = c.f64;
    return OQ_OK;
}
}
