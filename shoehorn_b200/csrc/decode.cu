// Decoders (quant.rs:383-537, quant_iq.rs:409-426, 565-585, 732-754,
// 944-998, 1159-1189) and the fused weighted-error pass of row_error
// (quant.rs:618-630) for sm_100a.
//
// Every decoder keeps the reference's operand order, e.g. Q4_K
// (d*sc)*q - dmin*m and IQ2 ((d*(0.5+s))*0.25*g)*sign, so decoded values are
// bit-identical to decode_row.
#include "decode.cuh"
#include "kernels.cuh"

namespace shc {

// Elementwise "encodings" (quant.rs:546-560) round-tripped to f32.
__device__ __forceinline__ float roundtrip_plain(uint32_t type, float x) {
    if (type == SHC_TYPE_F16) return f16_val(f16_bits(x));
    if (type == SHC_TYPE_BF16) return __uint_as_float(__float_as_uint(x) & 0xFFFF0000u);
    return x;
}

// ---------------------------------------------------------------------------
// decode kernel: one thread per 32-element sub-chunk
// ---------------------------------------------------------------------------
__global__ void decode_kernel(uint32_t type, const uint8_t *src, int64_t n_rows, int64_t ne0, float *dst,
                              int64_t be, int64_t bb) {
    const int64_t nsub_blk = be / 32;
    const int64_t blocks_per_row = ne0 / be;
    const int64_t total = n_rows * blocks_per_row * nsub_blk;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t blk = t / nsub_blk;  // global block index (rows contiguous)
        const int sub = (int)(t - blk * nsub_blk);
        float y[32];
        decode_sub32(type, src + blk * bb, sub, y);
        float *o = dst + blk * be + sub * 32;
#pragma unroll
        for (int j = 0; j < 32; j++) o[j] = y[j];
    }
}

__global__ void decode_plain_kernel(uint32_t type, const uint8_t *src, int64_t n, float *dst) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        if (type == SHC_TYPE_F32) {
            dst[i] = reinterpret_cast<const float *>(src)[i];
        } else {
            const uint16_t h = (uint16_t)(src[2 * i] | (src[2 * i + 1] << 8));
            dst[i] = type == SHC_TYPE_F16 ? f16_val(h) : bf16_bits_to_f32(h);
        }
    }
}

cudaError_t launch_decode(uint32_t type, const uint8_t *src, int64_t n_rows, int64_t ne0, float *dst, int num_sms,
                          cudaStream_t st) {
    const int64_t be = block_elems(type), bb = block_bytes(type);
    if (be == 1) {
        const int64_t n = n_rows * ne0;
        int64_t blocks = (n + 255) / 256;
        if (blocks > (int64_t)num_sms * 16) blocks = (int64_t)num_sms * 16;
        if (blocks < 1) blocks = 1;
        decode_plain_kernel<<<(unsigned)blocks, 256, 0, st>>>(type, src, n, dst);
        return cudaGetLastError();
    }
    const int64_t total = n_rows * (ne0 / 32);
    int64_t blocks = (total + 127) / 128;
    if (blocks > (int64_t)num_sms * 32) blocks = (int64_t)num_sms * 32;
    if (blocks < 1) blocks = 1;
    decode_kernel<<<(unsigned)blocks, 128, 0, st>>>(type, src, n_rows, ne0, dst, be, bb);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Weighted squared error (quant.rs:618-630): err = sum_i f64(w_i) * d * d with
// d = f64(x_i - x^_i), folded in element order.  The fold is order-dependent
// in f64, so one thread owns one (sampled row, candidate type); blockIdx.y
// selects the candidate so a warp never mixes types.
// ---------------------------------------------------------------------------
struct SseArgs {
    uint32_t types[32];
    const uint8_t *codes[32];
};

__global__ void __launch_bounds__(128) row_sse_kernel(SseArgs s, EncArgs a, double *err) {
    const int t = blockIdx.y;
    const uint32_t type = s.types[t];
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= a.n_rows) return;
    const int64_t ne0 = a.src.ne0;
    const float *imr = im_row(a.im, ne0, a.row0 + i * a.row_step);
    const int64_t be = block_elems(type), bb = block_bytes(type);
    double e = 0.0;
    if (be == 1) {
        for (int64_t c = 0; c < ne0; c += 8) {
            float xv[8], wv[8];
            load8(a.src, i, c, xv);
            if (imr) {
#pragma unroll
                for (int k = 0; k < 8; k++) wv[k] = __ldg(imr + c + k);
            }
#pragma unroll
            for (int k = 0; k < 8; k++) {
                const double w = imr ? (double)wv[k] : 1.0;
                const double d = (double)(xv[k] - roundtrip_plain(type, xv[k]));
                e += w * d * d;
            }
        }
    } else {
        const uint8_t *row_codes = s.codes[t] + i * (ne0 / be) * bb;
        const int nsub = (int)(be / 32);
        for (int64_t b = 0; b < ne0 / be; b++) {
            for (int sub = 0; sub < nsub; sub++) {
                float y[32];
                decode_sub32(type, row_codes + b * bb, sub, y);
                const int64_t c0 = b * be + sub * 32;
#pragma unroll
                for (int l = 0; l < 32; l += 8) {
                    float xv[8], wv[8];
                    load8(a.src, i, c0 + l, xv);
                    if (imr) {
                        const float4 *p = reinterpret_cast<const float4 *>(imr + c0 + l);
                        const float4 w0 = __ldg(p), w1 = __ldg(p + 1);
                        wv[0] = w0.x; wv[1] = w0.y; wv[2] = w0.z; wv[3] = w0.w;
                        wv[4] = w1.x; wv[5] = w1.y; wv[6] = w1.z; wv[7] = w1.w;
                    }
#pragma unroll
                    for (int k = 0; k < 8; k++) {
                        const double w = imr ? (double)wv[k] : 1.0;
                        const double d = (double)(xv[k] - y[l + k]);
                        e += w * d * d;
                    }
                }
            }
        }
    }
    err[(int64_t)t * a.n_rows + i] = e;
}

cudaError_t launch_row_sse(const uint32_t *types_host, int n_types, const uint8_t *const *codes_host, const EncArgs &a,
                           double *err, cudaStream_t st) {
    if (n_types < 1 || n_types > 32) return cudaErrorInvalidValue;
    SseArgs s;
    for (int t = 0; t < n_types; t++) {
        s.types[t] = types_host[t];
        s.codes[t] = codes_host[t];
    }
    dim3 grid((unsigned)((a.n_rows + 127) / 128), (unsigned)n_types);
    row_sse_kernel<<<grid, 128, 0, st>>>(s, a, err);
    return cudaGetLastError();
}

}  // namespace shc
