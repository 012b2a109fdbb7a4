// Allocation-free encode entry point (shc_encode_rows_noalloc).
//
// For callers that cannot allocate device memory where they encode: the
// per-row sigma^2 scratch of the K-quant encoders lives in a fixed buffer
// compiled into the library instead of coming from cudaMallocAsync.  The
// kernels are the same ones shc_encode_rows launches, so the bytes are the
// same.
#include <mutex>

#include "kernels.cuh"
#include "shoehorn_cuda.h"

namespace {

constexpr int64_t kMaxRows = SHC_NOALLOC_MAX_ROWS;
constexpr int kMaxDevices = 64;

// One sigma^2 slot per row; every GPU that loads the library holds it.  Host
// code must not pass this name to a kernel (on the host it is only a
// stand-in): the device address is looked up below.
static __device__ __align__(256) float g_sigma2_scratch[kMaxRows];

float *g_scratch_addr[kMaxDevices] = {};
int g_num_sms[kMaxDevices] = {};
std::mutex g_setup_mu;

// Once per device, with that device current: resolve the buffer's device
// address and the SM count used to size the grids.
int setup_device(int dev, float **addr, int *sms) {
    std::lock_guard<std::mutex> lk(g_setup_mu);
    if (!g_scratch_addr[dev]) {
        float *p = nullptr;
        if (cudaGetSymbolAddress((void **)&p, g_sigma2_scratch) != cudaSuccess || !p) {
            cudaGetLastError();
            return SHC_ECUDA;
        }
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            return SHC_ECUDA;
        }
        g_num_sms[dev] = n;
        g_scratch_addr[dev] = p;
    }
    *addr = g_scratch_addr[dev];
    *sms = g_num_sms[dev];
    return SHC_OK;
}

}  // namespace

extern "C" int shc_encode_rows_noalloc(uint32_t type, uint32_t src_type, const void *src, int64_t n_rows,
                                       int64_t ne0, const float *im, int64_t im_len, int64_t rows_per_mat,
                                       int64_t row0, uint8_t *dst, void *stream) {
    if (type != SHC_TYPE_Q4_K && type != SHC_TYPE_Q5_K && type != SHC_TYPE_Q6_K) return SHC_EINVAL;
    if (src_type != SHC_SRC_F32 && src_type != SHC_SRC_F16 && src_type != SHC_SRC_BF16) return SHC_EINVAL;
    if (n_rows < 0 || ne0 <= 0 || ne0 % 256 != 0 || rows_per_mat < 0 || row0 < 0) return SHC_EINVAL;
    if (n_rows > kMaxRows) return SHC_ETOOLARGE;
    if (n_rows == 0) return SHC_OK;
    if (!src || !dst || ((uintptr_t)src & 15) != 0 || (im && ((uintptr_t)im & 15) != 0)) return SHC_EINVAL;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        return SHC_ENODEV;
    }
    float *sig = nullptr;
    int sms = 0;
    int rc = setup_device(dev, &sig, &sms);
    if (rc != SHC_OK) return rc;

    const int64_t rb = ne0 / 256 * shc::block_bytes(type);
    shc::EncArgs a{};
    a.src.ptr = src;
    a.src.src_type = (int)src_type;
    a.src.ne0 = ne0;
    a.src.row_stride = ne0;
    a.im.ptr = im;
    a.im.len = im ? im_len : 0;
    a.im.rows_per_mat = rows_per_mat;
    a.n_rows = n_rows;
    a.row0 = row0;
    a.row_step = 1;
    a.sigma2 = sig;
    a.dst = dst;
    a.dst_row_bytes = rb;
    a.status = nullptr;  // these encoders raise no device-side status
    a.dst_aligned16 = (((uintptr_t)dst & 15) == 0 && (rb & 15) == 0) ? 1 : 0;
    cudaStream_t st = (cudaStream_t)stream;
    cudaError_t e = shc::launch_row_sigma2(a.src, n_rows, sig, st);
    if (e == cudaSuccess) e = shc::launch_kquant(type, a, sms, st);
    return e == cudaSuccess ? SHC_OK : SHC_ECUDA;
}
