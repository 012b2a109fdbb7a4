// C ABI of the library (include/shoehorn_cuda.h): validation, stream-ordered
// scratch, launches, bounded waits and the pipelined host-buffer entry points.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <atomic>
#include <chrono>
#include <cstring>
#include <mutex>
#include <new>
#include <thread>
#include <vector>

#include "iq_host.h"
#include "kernels.cuh"
#include "shoehorn_cuda.h"

using namespace shc;

struct shc_ctx {
    int device = 0;
    int num_sms = 0;
    int *d_status = nullptr;
    int *h_status_pool = nullptr;  // pinned, kStatusSlots ints
    std::atomic<unsigned> status_slot{0};
    void *d_tables = nullptr;
    IqTables iq{};
    cudaMemPool_t pool = nullptr;  // per-call scratch; keeps its memory between calls
    std::atomic<int64_t> launches{0};
    // host-buffer pipeline resources (one host call at a time)
    std::mutex host_mu;
    static constexpr int kHostStreams = 5;
    cudaStream_t hs[kHostStreams] = {};  // h2d, compute, d2h, row sigma^2, second compute
    static constexpr int kHostEvents = 13;                       // the host-buffer encode's events, kept
    cudaEvent_t hev[kHostEvents] = {};
    static constexpr int kPinSlots = 6;  // pageable staging: in 0-2, out 3-5
    void *pin[kPinSlots] = {};
    size_t pin_bytes[kPinSlots] = {};
};

namespace {

constexpr unsigned kStatusSlots = 64;

struct DevGuard {
    int prev = -1;
    explicit DevGuard(int d) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != d) cudaSetDevice(d);
    }
    ~DevGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

int cuda_status(cudaError_t e) {
    if (e == cudaSuccess) return SHC_OK;
    if (getenv("SHC_DEBUG")) fprintf(stderr, "shoehorn_cuda: %s\n", cudaGetErrorString(e));
    if (e == cudaErrorMemoryAllocation) return SHC_ENOMEM;
    return SHC_ECUDA;
}

#define SHC_TRY(expr)                                   \
    do {                                                \
        cudaError_t _e = (expr);                        \
        if (_e != cudaSuccess) return cuda_status(_e);  \
    } while (0)

bool valid_src_type(uint32_t s) { return s == SHC_SRC_F32 || s == SHC_SRC_F16 || s == SHC_SRC_BF16; }
size_t src_elem_bytes(uint32_t s) { return s == SHC_SRC_F32 ? 4 : 2; }

bool encodable(uint32_t t) {
    switch (t) {
    case SHC_TYPE_F32: case SHC_TYPE_F16: case SHC_TYPE_BF16: case SHC_TYPE_Q8_0: case SHC_TYPE_Q4_K:
    case SHC_TYPE_Q5_K: case SHC_TYPE_Q6_K: case SHC_TYPE_Q4_0: case SHC_TYPE_Q4_1: case SHC_TYPE_Q5_0:
    case SHC_TYPE_Q5_1: case SHC_TYPE_Q2_K: case SHC_TYPE_Q3_K:
        return true;
    default:
        return is_iq(t) ? iq_supported(t) : false;
    }
}

// Wait for an event with a deadline; never blocks past it.  The first
// 200 us poll between yields (a 20 us sleep lasts ~70 us with Linux's
// default timer slack, which short waits such as a status read would pay in
// full); longer waits then poll every 20 us asleep.
int wait_event(cudaEvent_t ev, std::chrono::steady_clock::time_point deadline, bool bounded) {
    const auto spin_until = std::chrono::steady_clock::now() + std::chrono::microseconds(200);
    for (;;) {
        cudaError_t e = cudaEventQuery(ev);
        if (e == cudaSuccess) return SHC_OK;
        if (e != cudaErrorNotReady) return cuda_status(e);
        const auto now = std::chrono::steady_clock::now();
        if (bounded && now > deadline) return SHC_ETIMEOUT;
        if (now < spin_until) std::this_thread::yield();
        else std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

int wait_stream(cudaStream_t st, int64_t timeout_ms) {
    cudaEvent_t ev;
    SHC_TRY(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    cudaError_t e = cudaEventRecord(ev, st);
    if (e != cudaSuccess) {
        cudaEventDestroy(ev);
        return cuda_status(e);
    }
    auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms < 0 ? 0 : timeout_ms);
    int rc = wait_event(ev, deadline, timeout_ms >= 0);
    cudaEventDestroy(ev);
    return rc;
}

EncArgs make_args(shc_ctx *ctx, uint32_t src_type, const void *src, int64_t n_rows, int64_t ne0, int64_t row_stride,
                  const float *im, int64_t im_len, int64_t rows_per_mat, int64_t row0, int64_t row_step, uint8_t *dst,
                  int64_t dst_row_bytes) {
    EncArgs a{};
    a.src.ptr = src;
    a.src.src_type = (int)src_type;
    a.src.ne0 = ne0;
    a.src.row_stride = row_stride;
    a.im.ptr = im;
    a.im.len = im ? im_len : 0;
    a.im.rows_per_mat = rows_per_mat;
    a.n_rows = n_rows;
    a.row0 = row0;
    a.row_step = row_step;
    a.sigma2 = nullptr;
    a.dst = dst;
    a.dst_row_bytes = dst_row_bytes;
    a.status = ctx->d_status;
    a.dst_aligned16 = (((uintptr_t)dst & 15) == 0 && (dst_row_bytes & 15) == 0) ? 1 : 0;
    return a;
}

int check_common(shc_ctx *ctx, uint32_t src_type, const void *src, int64_t n_rows, int64_t ne0, const float *im,
                 int64_t rows_per_mat, int64_t row0) {
    if (!ctx) return SHC_EINVAL;
    if (!valid_src_type(src_type) || n_rows < 0 || ne0 <= 0) return SHC_EINVAL;
    // global row indices and matrix heights are unsigned in the reference
    // (imatrix.rs:124 row_slice takes usize); a negative one would select a
    // matrix before the imatrix
    if (rows_per_mat < 0 || row0 < 0) return SHC_EINVAL;
    if (n_rows > 0 && !src) return SHC_EINVAL;
    if (((uintptr_t)src & 15) != 0) return SHC_EINVAL;  // 128-bit row loads
    if (im && ((uintptr_t)im & 15) != 0) return SHC_EINVAL;
    return SHC_OK;
}

// Stream-ordered per-call scratch from the context's pool.
cudaError_t scratch_alloc(shc_ctx *ctx, void **p, size_t bytes, cudaStream_t st) {
    return cudaMallocFromPoolAsync(p, bytes, ctx->pool, st);
}

// Encode one view of rows on `st` (sigma^2 pre-pass into stream-ordered
// scratch when the type needs it).
// sms: SMs the encoder's persistent grid is sized for (0: all of them).
int encode_view(shc_ctx *ctx, uint32_t type, EncArgs a, cudaStream_t st, int sms = 0) {
    const int num_sms = sms > 0 ? sms : ctx->num_sms;
    if (a.n_rows == 0) return SHC_OK;
    float *sig = nullptr;
    if (needs_sigma2(type) && !a.sigma2) {  // a caller may have computed it already
        SHC_TRY(scratch_alloc(ctx, (void **)&sig, sizeof(float) * (size_t)a.n_rows, st));
        cudaError_t e = launch_row_sigma2(a.src, a.n_rows, sig, st);
        ctx->launches++;
        if (e != cudaSuccess) {
            cudaFreeAsync(sig, st);
            return cuda_status(e);
        }
        a.sigma2 = sig;
    }
    cudaError_t e;
    if (block_elems(type) == 1) e = launch_plain(type, a, num_sms, st);
    else if (is_iq(type)) e = launch_iq(type, a, ctx->iq, num_sms, st);
    else e = launch_kquant(type, a, num_sms, st);
    ctx->launches++;
    if (sig) cudaFreeAsync(sig, st);
    return cuda_status(e);
}

// Re-encode the host lists (quant_iq.rs neighbour order kept) into the layout
// the device encoders read.  Every list is scanned in groups of four
// entries: its entries start on a four-entry boundary and are padded to a
// multiple of four with copies of the list's last entry (a later copy never
// wins: the scans keep the first of equal distances).  IQ2_XXS entries are
// 8-bit grid indices (lists of at most 255), the others 16-bit packed
// coordinates.  An off-grid kmap entry carries both the list's first entry
// and its length: kmap = -(1 + offset + (count << kListCountShift)).
constexpr int kListCountShift = 19;
void device_lists(int w, const IqHostTable &t, std::vector<int32_t> &kmap, std::vector<uint8_t> &bytes) {
    kmap = t.kmap;
    bytes.clear();
    const size_t esz = w == 0 ? 1 : 2;
    auto put = [&](size_t slot, uint32_t v) {
        if ((slot + 1) * esz > bytes.size()) bytes.resize((slot + 1) * esz, 0);
        if (esz == 1) bytes[slot] = (uint8_t)v;
        else reinterpret_cast<uint16_t *>(bytes.data())[slot] = (uint16_t)v;
    };
    for (size_t c = 0; c < t.kmap.size(); c++) {
        const int32_t m = t.kmap[c];
        if (m >= 0) continue;
        const size_t off = (size_t)(-m - 1);
        const uint32_t n = t.neighbours[off];
        auto entry = [&](uint32_t k) {  // k-th entry of the list, 1-based
            const uint32_t e = t.neighbours[off + k];
            return w == 0 ? (e & 0xFFFF) : (e >> 16);
        };
        const size_t slot = (bytes.size() / esz + 3) / 4 * 4;
        const uint32_t padded = (n + 3) / 4 * 4;
        for (uint32_t k = 1; k <= padded; k++) put(slot + k - 1, entry(k <= n ? k : n));
        if (n == 0 || n >= (1u << (31 - kListCountShift)) || slot >= (1u << kListCountShift)) {
            kmap.clear();  // the encoding cannot hold it (never at the shipped grids)
            return;
        }
        kmap[c] = -(int32_t)(1 + slot + ((size_t)n << kListCountShift));
    }
    while (bytes.size() % 16) bytes.push_back(0);
}

int upload_iq_tables(shc_ctx *ctx) {
    IqHostTable t[5];
    std::vector<int32_t> dk[5];
    std::vector<uint8_t> lists[5];
    size_t total = 0;
    for (int w = 0; w < 5; w++) {
        build_iq_tables(w, t[w]);
        device_lists(w, t[w], dk[w], lists[w]);
        if (dk[w].empty()) return SHC_EINVAL;
        total += (t[w].kmap.size() * 2 + t[w].neighbours.size() + t[w].grid_coords.size()) * 4 + lists[w].size() + 1024;
    }
    SHC_TRY(cudaMalloc(&ctx->d_tables, total));
    std::vector<uint8_t> host(total, 0);
    size_t off = 0;
    auto place = [&](const void *p, size_t bytes) {
        std::memcpy(host.data() + off, p, bytes);
        size_t at = off;
        off += (bytes + 255) & ~(size_t)255;
        return static_cast<uint8_t *>(ctx->d_tables) + at;
    };
    for (int w = 0; w < 5; w++) {
        ctx->iq.kmap[w] = reinterpret_cast<const int32_t *>(place(t[w].kmap.data(), t[w].kmap.size() * 4));
        ctx->iq.neighbours[w] = reinterpret_cast<const uint32_t *>(place(t[w].neighbours.data(), t[w].neighbours.size() * 4));
        ctx->iq.grid_coords[w] = reinterpret_cast<const uint32_t *>(place(t[w].grid_coords.data(), t[w].grid_coords.size() * 4));
        ctx->iq.dkmap[w] = reinterpret_cast<const int32_t *>(place(dk[w].data(), dk[w].size() * 4));
        ctx->iq.lists[w] = place(lists[w].data(), lists[w].size());
        ctx->iq.lists_bytes[w] = (int)lists[w].size();
    }
    SHC_TRY(cudaMemcpy(ctx->d_tables, host.data(), total, cudaMemcpyHostToDevice));
    return SHC_OK;
}

int ensure_pinned(shc_ctx *ctx, int slot, size_t bytes) {
    if (ctx->pin_bytes[slot] >= bytes) return SHC_OK;
    if (ctx->pin[slot]) cudaFreeHost(ctx->pin[slot]);
    ctx->pin[slot] = nullptr;
    ctx->pin_bytes[slot] = 0;
    SHC_TRY(cudaHostAlloc(&ctx->pin[slot], bytes, cudaHostAllocDefault));
    ctx->pin_bytes[slot] = bytes;
    return SHC_OK;
}

bool is_pinned(const void *p) {
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return attr.type == cudaMemoryTypeHost;
}

}  // namespace

extern "C" {

const char *shc_status_string(int s) {
    switch (s) {
    case SHC_OK: return "ok";
    case SHC_EINVAL: return "invalid argument";
    case SHC_ECUDA: return "CUDA runtime error";
    case SHC_EOFFGRID: return "IQ point off the lattice";
    case SHC_ENONEIGHBOUR: return "IQ neighbour search found no finite candidate";
    case SHC_ETIMEOUT: return "timed out";
    case SHC_ENOMEM: return "out of memory";
    case SHC_ENODEV: return "no usable sm_100 device";
    case SHC_ETOOLARGE: return "request exceeds the fixed scratch of shc_encode_rows_noalloc";
    default: return "unknown status";
    }
}

int64_t shc_row_bytes(uint32_t type, int64_t ne0) {
    const int64_t be = block_elems(type), bb = block_bytes(type);
    if (be == 0 || ne0 < 0 || ne0 % be != 0) return -1;
    return ne0 / be * bb;
}

int shc_type_supported(uint32_t type) { return encodable(type) ? 1 : 0; }

int shc_init(int device, shc_ctx **out) {
    if (!out) return SHC_EINVAL;
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
        cudaGetLastError();
        return SHC_ENODEV;
    }
    cudaDeviceProp prop;
    SHC_TRY(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10) return SHC_ENODEV;  // built for sm_100a only
    DevGuard g(device);
    shc_ctx *ctx = new (std::nothrow) shc_ctx();
    if (!ctx) return SHC_ENOMEM;
    ctx->device = device;
    ctx->num_sms = prop.multiProcessorCount;
    int rc = SHC_OK;
    if (cudaMalloc((void **)&ctx->d_status, sizeof(int)) != cudaSuccess ||
        cudaMemset(ctx->d_status, 0, sizeof(int)) != cudaSuccess ||
        cudaHostAlloc((void **)&ctx->h_status_pool, sizeof(int) * kStatusSlots, cudaHostAllocDefault) != cudaSuccess) {
        rc = SHC_ENOMEM;
    }
    if (rc == SHC_OK) {
        cudaMemPoolProps pp{};
        pp.allocType = cudaMemAllocationTypePinned;
        pp.handleTypes = cudaMemHandleTypeNone;
        pp.location.type = cudaMemLocationTypeDevice;
        pp.location.id = device;
        uint64_t keep = UINT64_MAX;  // never hand memory back at a synchronisation
        if (cudaMemPoolCreate(&ctx->pool, &pp) != cudaSuccess ||
            cudaMemPoolSetAttribute(ctx->pool, cudaMemPoolAttrReleaseThreshold, &keep) != cudaSuccess)
            rc = SHC_ECUDA;
    }
    if (rc == SHC_OK) rc = upload_iq_tables(ctx);
    for (int i = 0; rc == SHC_OK && i < shc_ctx::kHostStreams; i++)
        if (cudaStreamCreateWithFlags(&ctx->hs[i], cudaStreamNonBlocking) != cudaSuccess) rc = SHC_ECUDA;
    for (int i = 0; rc == SHC_OK && i < shc_ctx::kHostEvents; i++)
        if (cudaEventCreateWithFlags(&ctx->hev[i], cudaEventDisableTiming) != cudaSuccess) rc = SHC_ECUDA;
    if (rc != SHC_OK) {
        shc_free(ctx);
        return rc;
    }
    *out = ctx;
    return SHC_OK;
}

int shc_free(shc_ctx *ctx) {
    if (!ctx) return SHC_EINVAL;
    {
        DevGuard g(ctx->device);
        cudaDeviceSynchronize();
        for (int i = 0; i < shc_ctx::kHostStreams; i++)
            if (ctx->hs[i]) cudaStreamDestroy(ctx->hs[i]);
        for (int i = 0; i < shc_ctx::kHostEvents; i++)
            if (ctx->hev[i]) cudaEventDestroy(ctx->hev[i]);
        for (int i = 0; i < shc_ctx::kPinSlots; i++)
            if (ctx->pin[i]) cudaFreeHost(ctx->pin[i]);
        if (ctx->d_tables) cudaFree(ctx->d_tables);
        if (ctx->pool) cudaMemPoolDestroy(ctx->pool);
        if (ctx->d_status) cudaFree(ctx->d_status);
        if (ctx->h_status_pool) cudaFreeHost(ctx->h_status_pool);
    }
    delete ctx;
    return SHC_OK;
}

int64_t shc_launch_count(const shc_ctx *ctx) { return ctx ? ctx->launches.load() : -1; }

int shc_encode_rows(shc_ctx *ctx, uint32_t type, uint32_t src_type, const void *src, int64_t n_rows, int64_t ne0,
                    const float *im, int64_t im_len, int64_t rows_per_mat, int64_t row0, uint8_t *dst, void *stream) {
    int rc = check_common(ctx, src_type, src, n_rows, ne0, im, rows_per_mat, row0);
    if (rc != SHC_OK) return rc;
    const int64_t rb = shc_row_bytes(type, ne0);
    if (rb < 0 || !encodable(type) || (n_rows > 0 && !dst)) return SHC_EINVAL;
    if (block_elems(type) > 1 && ne0 % 8 != 0) return SHC_EINVAL;  // 128-bit row loads
    DevGuard g(ctx->device);
    EncArgs a = make_args(ctx, src_type, src, n_rows, ne0, ne0, im, im_len, rows_per_mat, row0, 1, dst, rb);
    return encode_view(ctx, type, a, (cudaStream_t)stream);
}

int shc_decode_rows(shc_ctx *ctx, uint32_t type, const uint8_t *src, int64_t n_rows, int64_t ne0, float *dst,
                    void *stream) {
    if (!ctx || n_rows < 0 || ne0 <= 0) return SHC_EINVAL;
    const int64_t rb = shc_row_bytes(type, ne0);
    if (rb < 0 || block_elems(type) == 0) return SHC_EINVAL;
    if (n_rows == 0) return SHC_OK;
    if (!src || !dst) return SHC_EINVAL;
    if (type == SHC_TYPE_F32 && ((uintptr_t)src & 3)) return SHC_EINVAL;
    DevGuard g(ctx->device);
    cudaError_t e = launch_decode(type, src, n_rows, ne0, dst, ctx->num_sms, (cudaStream_t)stream);
    ctx->launches++;
    return cuda_status(e);
}

int shc_row_errors(shc_ctx *ctx, const uint32_t *types, int n_types, uint32_t src_type, const void *src,
                   int64_t n_rows, int64_t ne0, const float *im, int64_t im_len, int64_t rows_per_mat, int64_t row0,
                   int64_t row_step, double *err, void *stream) {
    int rc = check_common(ctx, src_type, src, n_rows, ne0, im, rows_per_mat, row0);
    if (rc != SHC_OK) return rc;
    if (!types || n_types < 1 || n_types > 32 || row_step < 1) return SHC_EINVAL;
    for (int t = 0; t < n_types; t++)
        if (!encodable(types[t]) || shc_row_bytes(types[t], ne0) < 0) return SHC_EINVAL;
    const int64_t n_s = (n_rows + row_step - 1) / row_step;
    if (n_s == 0) return SHC_OK;
    if (!err) return SHC_EINVAL;
    DevGuard g(ctx->device);
    cudaStream_t st = (cudaStream_t)stream;
    EncArgs a = make_args(ctx, src_type, src, n_s, ne0, ne0 * row_step, im, im_len, rows_per_mat, row0, row_step,
                          nullptr, 0);
    bool any_sig = false;
    for (int t = 0; t < n_types; t++) any_sig |= needs_sigma2(types[t]);
    float *sig = nullptr;
    if (any_sig) {
        if (scratch_alloc(ctx, (void **)&sig, sizeof(float) * (size_t)n_s, st) != cudaSuccess) return SHC_ENOMEM;
        cudaError_t e = launch_row_sigma2(a.src, n_s, sig, st);
        ctx->launches++;
        if (e != cudaSuccess) {
            cudaFreeAsync(sig, st);
            return cuda_status(e);
        }
    }
    // One fused launch per candidate: encode, decode and the weighted
    // squared error in one kernel, the codes kept in shared memory (an
    // elementwise candidate round-trips each element in place of a code).
    cudaError_t e = cudaSuccess;
    for (int t = 0; t < n_types && e == cudaSuccess; t++) {
        const uint32_t ty = types[t];
        EncArgs at = a;
        at.sigma2 = sig;
        at.err = err + (size_t)t * (size_t)n_s;
        if (is_iq(ty)) e = launch_iq_fused(ty, at, ctx->iq, ctx->num_sms, st);
        else e = launch_kquant_fused(ty, at, ctx->num_sms, st);
        ctx->launches++;
    }
    if (sig) cudaFreeAsync(sig, st);
    return cuda_status(e);
}

int shc_sync(shc_ctx *ctx, void *stream, int64_t timeout_ms) {
    if (!ctx) return SHC_EINVAL;
    DevGuard g(ctx->device);
    cudaStream_t st = (cudaStream_t)stream;
    int *slot = ctx->h_status_pool + (ctx->status_slot.fetch_add(1) % kStatusSlots);
    *slot = 0;
    SHC_TRY(cudaMemcpyAsync(slot, ctx->d_status, sizeof(int), cudaMemcpyDeviceToHost, st));
    SHC_TRY(cudaMemsetAsync(ctx->d_status, 0, sizeof(int), st));
    int rc = wait_stream(st, timeout_ms);
    if (rc != SHC_OK) return rc;
    return *slot;
}

int shc_encode_tensor_host(shc_ctx *ctx, uint32_t type, uint32_t src_type, const void *host_src, int64_t n_rows,
                           int64_t ne0, const float *host_im, int64_t im_len, int64_t rows_per_mat, int64_t row0,
                           uint8_t *host_dst, int64_t timeout_ms) {
    if (!ctx || !valid_src_type(src_type) || n_rows < 0 || ne0 <= 0 || ne0 % 8 != 0) return SHC_EINVAL;
    if (rows_per_mat < 0 || row0 < 0) return SHC_EINVAL;
    const int64_t rb = shc_row_bytes(type, ne0);
    if (rb < 0 || !encodable(type)) return SHC_EINVAL;
    if (n_rows == 0) return SHC_OK;
    if (!host_src || !host_dst) return SHC_EINVAL;
    std::lock_guard<std::mutex> lk(ctx->host_mu);
    DevGuard g(ctx->device);
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms < 0 ? 0 : timeout_ms);
    const bool bounded = timeout_ms >= 0;
    const size_t eb = src_elem_bytes(src_type);
    const size_t in_row = (size_t)ne0 * eb;
    // Chunks: equal chunks of at most ~16 MiB of source (a short tail chunk
    // would pay a whole row sigma^2 pass, a fixed serial-chain latency, for a
    // few rows), the last one cut in two so that less work is left once the
    // final host-to-device copy lands.  Three buffer slots: the copy of chunk
    // k+2 never waits for the encode of chunk k.
    constexpr int NS = 3;
    const int64_t max_chunk = std::max<int64_t>(1, (int64_t)((16u << 20) / in_row));
    const int64_t n_eq = (n_rows + max_chunk - 1) / max_chunk;
    const int64_t chunk = (n_rows + n_eq - 1) / n_eq;
    std::vector<std::pair<int64_t, int64_t>> chunks;  // (first row, rows)
    for (int64_t r = 0; r < n_rows; r += chunk) chunks.emplace_back(r, std::min(chunk, n_rows - r));
    if (n_eq > 1 && chunks.back().second >= 64) {
        const auto last = chunks.back();
        const int64_t h = last.second / 2;
        chunks.back().second = last.second - h;
        chunks.emplace_back(last.first + last.second - h, h);
    }
    const int64_t n_chunks = (int64_t)chunks.size();
    const bool pin_src = is_pinned(host_src), pin_dst = is_pinned(host_dst);
    cudaStream_t s_in = ctx->hs[0], s_cmp = ctx->hs[1], s_out = ctx->hs[2], s_sig = ctx->hs[3], s_cmp2 = ctx->hs[4];
    // The row sigma^2 pre-pass (one thread per row, bound by its serial sums)
    // runs on its own stream for chunk k+1 while chunk k encodes; the
    // encoder's persistent grid leaves kSigmaSms SMs' worth of blocks free so
    // that the pre-pass has room beside it.
    constexpr int kSigmaSms = 4;
    const bool pre_sig = needs_sigma2(type) && n_rows > 1;
    const int enc_sms = pre_sig ? std::max(1, ctx->num_sms - kSigmaSms) : 0;
    // Without the pre-pass, consecutive chunks encode on two streams in
    // turn: each encoder's persistent grid ends with its slowest warps'
    // last units (about one unit's time, 0.2 ms for the IQ2 encoders), and
    // the next chunk's blocks take the SMs as they free up.  (The pre-pass
    // types keep one stream: a second encoder would take the SMs the
    // pre-pass of the next chunk runs on.)
    const bool two_cmp = !pre_sig;
    int rc = SHC_OK;
    void *d_in[NS] = {};
    uint8_t *d_out[NS] = {};
    float *d_sig[NS] = {};
    float *d_im = nullptr;
    // the context's events (one host-buffer call at a time holds host_mu)
    static_assert(4 * NS + 1 <= shc_ctx::kHostEvents, "host events");
    cudaEvent_t *ev_in = ctx->hev, *ev_cmp = ctx->hev + NS, *ev_out = ctx->hev + 2 * NS, *ev_sig = ctx->hev + 3 * NS;
    auto fail = [&](int code) {
        if (rc == SHC_OK) rc = code;
    };
    const int nslots = (int)std::min<int64_t>(NS, n_chunks);
    for (int b = 0; b < nslots && rc == SHC_OK; b++) {
        if (scratch_alloc(ctx, &d_in[b], in_row * (size_t)chunk, s_cmp) != cudaSuccess) fail(SHC_ENOMEM);
        if (scratch_alloc(ctx, (void **)&d_out[b], (size_t)rb * (size_t)chunk, s_cmp) != cudaSuccess) fail(SHC_ENOMEM);
        if (pre_sig && rc == SHC_OK &&
            scratch_alloc(ctx, (void **)&d_sig[b], sizeof(float) * (size_t)chunk, s_cmp) != cudaSuccess)
            fail(SHC_ENOMEM);
        if (!pin_src && rc == SHC_OK) fail(ensure_pinned(ctx, b, in_row * (size_t)chunk));
        if (!pin_dst && rc == SHC_OK) fail(ensure_pinned(ctx, NS + b, (size_t)rb * (size_t)chunk));
    }
    if (rc == SHC_OK && host_im && im_len > 0) {
        if (scratch_alloc(ctx, (void **)&d_im, sizeof(float) * (size_t)im_len, s_cmp) != cudaSuccess) fail(SHC_ENOMEM);
        else if (cudaMemcpyAsync(d_im, host_im, sizeof(float) * (size_t)im_len, cudaMemcpyHostToDevice, s_cmp) != cudaSuccess)
            fail(SHC_ECUDA);
    }
    if (rc == SHC_OK) {
        // the allocations above are ordered on s_cmp; make the other streams wait
        cudaEventRecord(ev_cmp[0], s_cmp);
        cudaStreamWaitEvent(s_in, ev_cmp[0], 0);
        cudaStreamWaitEvent(s_out, ev_cmp[0], 0);
        cudaStreamWaitEvent(s_sig, ev_cmp[0], 0);
        cudaStreamWaitEvent(s_cmp2, ev_cmp[0], 0);
        for (int b = 0; b < NS; b++) {
            cudaEventRecord(ev_cmp[b], s_cmp);
            cudaEventRecord(ev_out[b], s_out);
            cudaEventRecord(ev_in[b], s_in);
        }
    }
    int64_t pending_out[NS];  // chunk whose pageable output sits in pin[NS + b]
    for (int b = 0; b < NS; b++) pending_out[b] = -1;
    auto drain_out = [&](int b) {
        if (pending_out[b] < 0) return;
        int w = wait_event(ev_out[b], deadline, bounded);
        if (w != SHC_OK) {
            fail(w);
            return;
        }
        const auto &c = chunks[(size_t)pending_out[b]];
        std::memcpy(host_dst + c.first * rb, ctx->pin[NS + b], (size_t)(c.second * rb));
        pending_out[b] = -1;
    };
    for (int64_t k = 0; k < n_chunks && rc == SHC_OK; k++) {
        const int b = (int)(k % NS);
        const int64_t r0 = chunks[(size_t)k].first, nr = chunks[(size_t)k].second;
        const size_t in_bytes = in_row * (size_t)nr;
        const uint8_t *src_k = static_cast<const uint8_t *>(host_src) + (size_t)r0 * in_row;
        // H2D of chunk k into d_in[b] once the encode of chunk k-NS released it
        cudaStreamWaitEvent(s_in, ev_cmp[b], 0);
        if (pin_src) {
            if (cudaMemcpyAsync(d_in[b], src_k, in_bytes, cudaMemcpyHostToDevice, s_in) != cudaSuccess) fail(SHC_ECUDA);
        } else {
            int w = wait_event(ev_in[b], deadline, bounded);  // staging slot free
            if (w != SHC_OK) { fail(w); break; }
            std::memcpy(ctx->pin[b], src_k, in_bytes);
            if (cudaMemcpyAsync(d_in[b], ctx->pin[b], in_bytes, cudaMemcpyHostToDevice, s_in) != cudaSuccess) fail(SHC_ECUDA);
        }
        cudaEventRecord(ev_in[b], s_in);
        EncArgs a = make_args(ctx, src_type, d_in[b], nr, ne0, ne0, d_im, im_len, rows_per_mat, row0 + r0, 1, d_out[b], rb);
        // sigma^2 of chunk k once its input landed (d_sig[b] is free: the
        // chunk's H2D already waited for the encode of chunk k-NS)
        cudaEvent_t ready = ev_in[b];
        if (pre_sig) {
            cudaStreamWaitEvent(s_sig, ev_in[b], 0);
            if (launch_row_sigma2(a.src, nr, d_sig[b], s_sig) != cudaSuccess) { fail(SHC_ECUDA); break; }
            ctx->launches++;
            cudaEventRecord(ev_sig[b], s_sig);
            ready = ev_sig[b];
            a.sigma2 = d_sig[b];
        }
        // encode chunk k once its input (and sigma^2) landed and d_out[b] was drained
        cudaStream_t sc = (two_cmp && (k & 1)) ? s_cmp2 : s_cmp;
        cudaStreamWaitEvent(sc, ready, 0);
        cudaStreamWaitEvent(sc, ev_out[b], 0);
        int e = encode_view(ctx, type, a, sc, enc_sms);
        if (e != SHC_OK) { fail(e); break; }
        cudaEventRecord(ev_cmp[b], sc);
        // D2H of chunk k
        cudaStreamWaitEvent(s_out, ev_cmp[b], 0);
        if (pin_dst) {
            if (cudaMemcpyAsync(host_dst + r0 * rb, d_out[b], (size_t)(nr * rb), cudaMemcpyDeviceToHost, s_out) != cudaSuccess)
                fail(SHC_ECUDA);
        } else {
            drain_out(b);
            if (cudaMemcpyAsync(ctx->pin[NS + b], d_out[b], (size_t)(nr * rb), cudaMemcpyDeviceToHost, s_out) != cudaSuccess)
                fail(SHC_ECUDA);
            pending_out[b] = k;
        }
        cudaEventRecord(ev_out[b], s_out);
    }
    for (int b = 0; b < NS; b++) drain_out(b);
    // release buffers after all queued work; wait (bounded) for completion
    cudaEvent_t done = ctx->hev[4 * NS];
    cudaEventRecord(done, s_in);
    cudaStreamWaitEvent(s_cmp, done, 0);
    cudaEventRecord(done, s_out);
    cudaStreamWaitEvent(s_cmp, done, 0);
    cudaEventRecord(done, s_sig);
    cudaStreamWaitEvent(s_cmp, done, 0);
    cudaEventRecord(done, s_cmp2);
    cudaStreamWaitEvent(s_cmp, done, 0);
    for (int b = 0; b < NS; b++) {
        if (d_in[b]) cudaFreeAsync(d_in[b], s_cmp);
        if (d_out[b]) cudaFreeAsync(d_out[b], s_cmp);
        if (d_sig[b]) cudaFreeAsync(d_sig[b], s_cmp);
    }
    if (d_im) cudaFreeAsync(d_im, s_cmp);
    // the device status word of this call's kernels, read and cleared behind
    // them (as shc_sync does), so that one wait covers both
    int *slot = ctx->h_status_pool + (ctx->status_slot.fetch_add(1) % kStatusSlots);
    *slot = 0;
    const bool status_read = rc == SHC_OK &&
                             cudaMemcpyAsync(slot, ctx->d_status, sizeof(int), cudaMemcpyDeviceToHost, s_cmp) == cudaSuccess &&
                             cudaMemsetAsync(ctx->d_status, 0, sizeof(int), s_cmp) == cudaSuccess;
    if (rc == SHC_OK && !status_read) rc = SHC_ECUDA;
    cudaEventRecord(done, s_cmp);
    int w = wait_event(done, deadline, bounded);
    if (rc == SHC_OK) rc = w;
    if (rc == SHC_OK && *slot != SHC_OK) rc = *slot;
    return rc;
}

int shc_row_errors_host(shc_ctx *ctx, const uint32_t *types, int n_types, uint32_t src_type, const void *host_src,
                        int64_t n_rows, int64_t ne0, const float *host_im, int64_t im_len, int64_t rows_per_mat,
                        int64_t row0, int64_t row_step, double *err, int64_t timeout_ms) {
    if (!ctx || !valid_src_type(src_type) || n_rows < 0 || ne0 <= 0 || row_step < 1 || !types || n_types < 1 ||
        n_types > 32 || rows_per_mat < 0 || row0 < 0)
        return SHC_EINVAL;
    const int64_t n_s = (n_rows + row_step - 1) / row_step;
    if (n_s == 0) return SHC_OK;
    if (!host_src || !err) return SHC_EINVAL;
    std::lock_guard<std::mutex> lk(ctx->host_mu);
    DevGuard g(ctx->device);
    cudaStream_t st = ctx->hs[1];
    const size_t eb = src_elem_bytes(src_type), in_row = (size_t)ne0 * eb;
    // sampled rows in chunks of ~256 MiB of source
    int64_t chunk = std::max<int64_t>(1, (int64_t)((256u << 20) / in_row));
    chunk = std::min(chunk, n_s);
    void *d_in = nullptr;
    float *d_im = nullptr;
    double *d_err = nullptr;
    int rc = SHC_OK;
    if (scratch_alloc(ctx, &d_in, in_row * (size_t)chunk, st) != cudaSuccess ||
        scratch_alloc(ctx, (void **)&d_err, sizeof(double) * (size_t)n_types * (size_t)chunk, st) != cudaSuccess)
        rc = SHC_ENOMEM;
    if (rc == SHC_OK && host_im && im_len > 0) {
        if (scratch_alloc(ctx, (void **)&d_im, sizeof(float) * (size_t)im_len, st) != cudaSuccess) rc = SHC_ENOMEM;
        else if (cudaMemcpyAsync(d_im, host_im, sizeof(float) * (size_t)im_len, cudaMemcpyHostToDevice, st) != cudaSuccess)
            rc = SHC_ECUDA;
    }
    std::vector<double> part((size_t)n_types * (size_t)chunk);
    for (int64_t i0 = 0; i0 < n_s && rc == SHC_OK; i0 += chunk) {
        const int64_t ni = std::min(chunk, n_s - i0);
        const uint8_t *src0 = static_cast<const uint8_t *>(host_src) + (size_t)(i0 * row_step) * in_row;
        // gather the sampled rows (pitch row_step rows) in one strided copy
        if (cudaMemcpy2DAsync(d_in, in_row, src0, in_row * (size_t)row_step, in_row, (size_t)ni, cudaMemcpyHostToDevice,
                              st) != cudaSuccess) {
            rc = SHC_ECUDA;
            break;
        }
        rc = shc_row_errors(ctx, types, n_types, src_type, d_in, ni, ne0, d_im, im_len, rows_per_mat,
                            row0 + i0 * row_step, 1, d_err, st);
        if (rc != SHC_OK) break;
        if (cudaMemcpyAsync(part.data(), d_err, sizeof(double) * (size_t)n_types * (size_t)ni, cudaMemcpyDeviceToHost,
                            st) != cudaSuccess) {
            rc = SHC_ECUDA;
            break;
        }
        rc = wait_stream(st, timeout_ms);
        if (rc != SHC_OK) break;
        for (int t = 0; t < n_types; t++)
            std::memcpy(err + (size_t)t * (size_t)n_s + (size_t)i0, part.data() + (size_t)t * (size_t)ni,
                        sizeof(double) * (size_t)ni);
    }
    if (d_in) cudaFreeAsync(d_in, st);
    if (d_err) cudaFreeAsync(d_err, st);
    if (d_im) cudaFreeAsync(d_im, st);
    int s = shc_sync(ctx, st, timeout_ms);
    return rc != SHC_OK ? rc : s;
}

int shc_grid_info(int which, int32_t *grid_size, int32_t *map_size, int64_t *n_neighbours, int32_t *map_out,
                  uint32_t *neighbours_out) {
    if (which < 0 || which > 4) return SHC_EINVAL;
    IqHostTable t;
    build_iq_tables(which, t);
    if (grid_size) *grid_size = t.grid_size;
    if (map_size) *map_size = (int32_t)t.kmap.size();
    if (n_neighbours) *n_neighbours = (int64_t)t.neighbours.size();
    if (map_out) std::memcpy(map_out, t.kmap.data(), t.kmap.size() * 4);
    if (neighbours_out) std::memcpy(neighbours_out, t.neighbours.data(), t.neighbours.size() * 4);
    return SHC_OK;
}

}  // extern "C"
