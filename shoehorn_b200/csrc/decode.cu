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

}  // namespace shc
