// FP32 issue-rate probe for the encoder roofline on sm_100.
//
// The encoders may not contract multiply-adds (their results must equal the
// reference's separately rounded f32 operations), so their ceiling is the
// rate of separate adds and multiplies, scalar or packed f32x2 (two f32
// operations per lane per instruction, issued at half the scalar rate).  This
// program times long independent chains of each form, a fused multiply-add
// for comparison, and the rounding and min/max forms the encoders use, and
// prints f32 operations per clock per SM at the device's reported maximum
// clock.  Packed chains are add-only or multiply-only: a packed multiply
// feeding a packed add can be contracted into FFMA2 by code generation.  Every kernel touches only registers and writes
// one float per thread.
#include <cstdio>
#include <cuda_runtime.h>

namespace {
constexpr int kChains = 8;
constexpr int kIters = 4096;

__global__ void scalar_mul_add(float *out, float a, float b) {
    float x[kChains];
    for (int i = 0; i < kChains; i++) x[i] = threadIdx.x * 1e-3f + i;
    for (int it = 0; it < kIters; it++)
#pragma unroll
        for (int i = 0; i < kChains; i++) x[i] = __fadd_rn(__fmul_rn(x[i], a), b);
    float s = 0.0f;
    for (int i = 0; i < kChains; i++) s += x[i];
    out[blockIdx.x * blockDim.x + threadIdx.x] = s;
}

// Add-only and multiply-only chains: nothing for the compiler to contract.
__global__ void packed_add(float *out, float a, float) {
    float2 x[kChains];
    for (int i = 0; i < kChains; i++) x[i] = make_float2(threadIdx.x * 1e-3f + i, i * 0.5f);
    const float2 A = make_float2(a, a);
    for (int it = 0; it < kIters; it++)
#pragma unroll
        for (int i = 0; i < kChains; i++) x[i] = __fadd2_rn(x[i], A);
    float s = 0.0f;
    for (int i = 0; i < kChains; i++) s += x[i].x + x[i].y;
    out[blockIdx.x * blockDim.x + threadIdx.x] = s;
}

__global__ void packed_mul(float *out, float a, float) {
    float2 x[kChains];
    for (int i = 0; i < kChains; i++) x[i] = make_float2(threadIdx.x * 1e-3f + i, i * 0.5f);
    const float2 A = make_float2(a, a);
    for (int it = 0; it < kIters; it++)
#pragma unroll
        for (int i = 0; i < kChains; i++) x[i] = __fmul2_rn(x[i], A);
    float s = 0.0f;
    for (int i = 0; i < kChains; i++) s += x[i].x + x[i].y;
    out[blockIdx.x * blockDim.x + threadIdx.x] = s;
}

// Fused multiply-add, for reference: the encoders may not use it.
__global__ void scalar_fma(float *out, float a, float b) {
    float x[kChains];
    for (int i = 0; i < kChains; i++) x[i] = threadIdx.x * 1e-3f + i;
    for (int it = 0; it < kIters; it++)
#pragma unroll
        for (int i = 0; i < kChains; i++) x[i] = __fmaf_rn(x[i], a, b);
    float s = 0.0f;
    for (int i = 0; i < kChains; i++) s += x[i];
    out[blockIdx.x * blockDim.x + threadIdx.x] = s;
}

__global__ void mul_roundf(float *out, float a, float) {
    float x[kChains];
    for (int i = 0; i < kChains; i++) x[i] = threadIdx.x * 1e-3f + i;
    for (int it = 0; it < kIters; it++)
#pragma unroll
        for (int i = 0; i < kChains; i++) x[i] = roundf(__fmul_rn(x[i], a));
    float s = 0.0f;
    for (int i = 0; i < kChains; i++) s += x[i];
    out[blockIdx.x * blockDim.x + threadIdx.x] = s;
}

__global__ void mul_add_rounding(float *out, float a, float) {
    float x[kChains];
    for (int i = 0; i < kChains; i++) x[i] = threadIdx.x * 1e-3f + i;
    for (int it = 0; it < kIters; it++)
#pragma unroll
        for (int i = 0; i < kChains; i++) {
            const float y = __fmul_rn(x[i], a);
            x[i] = __fadd_rn(__fadd_rd(__fadd_rz(y, 0.5f), 8388608.0f), -8388608.0f);
        }
    float s = 0.0f;
    for (int i = 0; i < kChains; i++) s += x[i];
    out[blockIdx.x * blockDim.x + threadIdx.x] = s;
}

__global__ void min_max(float *out, float a, float b) {
    float x[kChains];
    for (int i = 0; i < kChains; i++) x[i] = threadIdx.x * 1e-3f + i;
    for (int it = 0; it < kIters; it++)
#pragma unroll
        for (int i = 0; i < kChains; i++) x[i] = fminf(fmaxf(x[i] + 0.0f * it, a), b);
    float s = 0.0f;
    for (int i = 0; i < kChains; i++) s += x[i];
    out[blockIdx.x * blockDim.x + threadIdx.x] = s;
}
}  // namespace

int main() {
    int sms = 0, khz = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0) != cudaSuccess ||
        cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, 0) != cudaSuccess) {
        printf("no CUDA device\n");
        return 1;
    }
    const int blocks = sms * 8, threads = 256;
    float *out = nullptr;
    if (cudaMalloc(&out, sizeof(float) * blocks * threads) != cudaSuccess) return 1;
    struct Probe {
        const char *name;
        void (*fn)(float *, float, float);
        int ops;  // f32 operations per chain step (counted as the encoders' op counter does)
    } probes[] = {{"scalar mul + add", scalar_mul_add, 2},
                  {"packed f32x2 add", packed_add, 2},
                  {"packed f32x2 mul", packed_mul, 2},
                  {"scalar fma (2 flops)", scalar_fma, 2},
                  {"mul + roundf", mul_roundf, 2},
                  {"mul + 3-add exact rounding", mul_add_rounding, 2},
                  {"fmaxf + fminf", min_max, 2}};
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    printf("%d SMs, max SM clock %d MHz\n", sms, khz / 1000);
    for (const Probe &p : probes) {
        float ms = 0.0f;
        for (int rep = 0; rep < 3; rep++) {
            cudaEventRecord(e0);
            p.fn<<<blocks, threads>>>(out, 1.0000001f, 0.25f);
            cudaEventRecord(e1);
            cudaEventSynchronize(e1);
            cudaEventElapsedTime(&ms, e0, e1);
        }
        const double steps = (double)blocks * threads * kIters * kChains;
        const double per_clk_sm = steps * p.ops / (ms * 1e-3) / sms / (khz * 1e3);
        printf("%-28s %8.3f ms  %7.1f f32 ops/clk/SM\n", p.name, ms, per_clk_sm);
    }
    const cudaError_t err = cudaDeviceSynchronize();
    printf("status: %s\n", cudaGetErrorString(err));
    cudaFree(out);
    return err == cudaSuccess ? 0 : 1;
}
