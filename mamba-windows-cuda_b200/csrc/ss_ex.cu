// Input / output transforms of Mamba's block around the selective scan (not in the
// reference; the official Mamba scan takes them): delta_eff = softplus(delta + delta_bias)
// (or delta + delta_bias), and the gate out_z = y * silu(z). This file holds the
// element-wise kernels and the C entry points mwc_ss_fwd_ex / mwc_ss_bwd_ex, which run them
// around the forward / backward scans (the scan kernels themselves are unchanged).
//
// Element-wise work is HBM-bound: grid-stride loops over (rows = B*L) x D with the channel
// index inner, so consecutive threads touch consecutive channels. The dbias reduction is
// deterministic: fixed row chunks per CTA, partial sums in a workspace, then a fixed-order
// sum over chunks.
#include "mwc_b200.h"
#include "mwc_device.cuh"
#include "mwc_internal.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdint>
#include <cstdio>

namespace mwc {

__device__ __forceinline__ float softplus_f(float x) { return x <= 20.f ? log1pf(expf(x)) : x; }
__device__ __forceinline__ float sigmoid_f(float x) { return 1.f / (1.f + expf(-x)); }

constexpr int EX_THREADS = 256;
constexpr int EX_ROWS_PER_CHUNK = 256;   // rows of B*L summed per dbias partial

static unsigned ex_blocks(int64_t n) {
    return (unsigned)std::max<int64_t>(1, std::min<int64_t>((n + EX_THREADS - 1) / EX_THREADS, 148 * 16));
}

// delta_eff = f(delta + bias[d]), f = softplus or identity
template <typename T>
__global__ void delta_eff_kernel(const T* __restrict__ delta, const T* __restrict__ bias, int softplus,
                                 T* __restrict__ out, int64_t n, int64_t D) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        float x = to_f(delta[i]) + (bias != nullptr ? to_f(bias[i % D]) : 0.f);
        out[i] = from_f<T>(softplus ? softplus_f(x) : x);
    }
}

// out_z = y * z * sigmoid(z)
template <typename T>
__global__ void gate_fwd_kernel(const T* __restrict__ y, const T* __restrict__ z, T* __restrict__ out_z, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float zz = to_f(z[i]);
        out_z[i] = from_f<T>(to_f(y[i]) * zz * sigmoid_f(zz));
    }
}

// gy = dout * silu(z); dz = dout * y * silu'(z), silu'(z) = s (1 + z (1 - s)), s = sigmoid(z)
template <typename T>
__global__ void gate_bwd_kernel(const T* __restrict__ dout, const T* __restrict__ z, const T* __restrict__ y,
                                T* __restrict__ gy, T* __restrict__ dz, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float g = to_f(dout[i]), zz = to_f(z[i]);
        const float s = sigmoid_f(zz);
        gy[i] = from_f<T>(g * zz * s);
        dz[i] = from_f<T>(g * to_f(y[i]) * s * (1.f + zz * (1.f - s)));
    }
}

// In place: ddelta = ddelta_eff * f'(delta + bias) (f' = sigmoid for softplus, 1 otherwise);
// partial[chunk][d] = sum over the chunk's rows of the new ddelta (float32, rows in order).
template <typename T>
__global__ void ddelta_kernel(T* __restrict__ ddelta, const T* __restrict__ delta, const T* __restrict__ bias,
                              int softplus, float* __restrict__ partial, int64_t rows, int64_t D) {
    const int64_t d = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t chunk = blockIdx.y;
    if (d >= D) return;
    const float bd = bias != nullptr ? to_f(bias[d]) : 0.f;
    const int64_t r0 = chunk * EX_ROWS_PER_CHUNK;
    const int64_t r1 = rows < r0 + EX_ROWS_PER_CHUNK ? rows : r0 + EX_ROWS_PER_CHUNK;
    float acc = 0.f;
    for (int64_t r = r0; r < r1; ++r) {
        const int64_t i = r * D + d;
        float g = to_f(ddelta[i]);
        if (softplus) g *= sigmoid_f(to_f(delta[i]) + bd);
        if (softplus) ddelta[i] = from_f<T>(g);
        acc += g;
    }
    if (partial != nullptr) partial[chunk * D + d] = acc;
}

template <typename T>
__global__ void dbias_final_kernel(const float* __restrict__ partial, int64_t nchunk, int64_t D, T* __restrict__ dbias) {
    for (int64_t d = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; d < D; d += (int64_t)gridDim.x * blockDim.x) {
        float s = 0.f;
        for (int64_t c = 0; c < nchunk; ++c) s += partial[c * D + d];
        dbias[d] = from_f<T>(s);
    }
}

template <typename T>
static cudaError_t launch_delta_eff(const void* delta, const void* bias, int softplus, void* out, int64_t n,
                                    int64_t D, cudaStream_t s) {
    delta_eff_kernel<T><<<ex_blocks(n), EX_THREADS, 0, s>>>(static_cast<const T*>(delta), static_cast<const T*>(bias),
                                                            softplus, static_cast<T*>(out), n, D);
    return cudaGetLastError();
}
template <typename T>
static cudaError_t launch_gate_fwd(const void* y, const void* z, void* out_z, int64_t n, cudaStream_t s) {
    gate_fwd_kernel<T><<<ex_blocks(n), EX_THREADS, 0, s>>>(static_cast<const T*>(y), static_cast<const T*>(z),
                                                           static_cast<T*>(out_z), n);
    return cudaGetLastError();
}
template <typename T>
static cudaError_t launch_gate_bwd(const void* dout, const void* z, const void* y, void* gy, void* dz, int64_t n,
                                   cudaStream_t s) {
    gate_bwd_kernel<T><<<ex_blocks(n), EX_THREADS, 0, s>>>(static_cast<const T*>(dout), static_cast<const T*>(z),
                                                           static_cast<const T*>(y), static_cast<T*>(gy),
                                                           static_cast<T*>(dz), n);
    return cudaGetLastError();
}
template <typename T>
static cudaError_t launch_ddelta(void* ddelta, const void* delta, const void* bias, int softplus, float* partial,
                                 int64_t rows, int64_t D, void* dbias, cudaStream_t s) {
    const int64_t nchunk = (rows + EX_ROWS_PER_CHUNK - 1) / EX_ROWS_PER_CHUNK;
    dim3 grid((unsigned)((D + EX_THREADS - 1) / EX_THREADS), (unsigned)nchunk);
    ddelta_kernel<T><<<grid, EX_THREADS, 0, s>>>(static_cast<T*>(ddelta), static_cast<const T*>(delta),
                                                 static_cast<const T*>(bias), softplus, partial, rows, D);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || dbias == nullptr) return e;
    dbias_final_kernel<T><<<ex_blocks(D), EX_THREADS, 0, s>>>(partial, nchunk, D, static_cast<T*>(dbias));
    return cudaGetLastError();
}

#define MWC_EX_DISPATCH(fn, dtype, ...)                                              \
    ((dtype) == 2 ? fn<__nv_bfloat16>(__VA_ARGS__)                                   \
                  : (dtype) == 1 ? fn<__half>(__VA_ARGS__) : fn<float>(__VA_ARGS__))

static inline int64_t ex_align(int64_t x) { return (x + 255) / 256 * 256; }

static int ex_fail(int code, const char* fmt, ...) {
    char buf[256];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    return report_error(code, buf);
}

}  // namespace mwc

using namespace mwc;

extern "C" {

int64_t mwc_ss_fwd_ex_workspace_bytes(int64_t B, int64_t L, int64_t D, int dtype) {
    if (B <= 0 || L <= 0 || D <= 0) return 0;
    const int64_t es = dtype == MWC_F32 ? 4 : 2;
    return ex_align(B * L * D * es) + mwc_ss_fwd_workspace_bytes(B, L, D, dtype);
}

int mwc_ss_fwd_ex(const void* u, const void* delta, const void* A, const void* Bm, const void* Cm,
                  const void* Dv, const void* z, const void* delta_bias, int delta_softplus,
                  const void* h_prev, void* out, void* out_z, void* h_last, float* ckpt,
                  void* workspace, int64_t workspace_bytes, int64_t B, int64_t L, int64_t D,
                  int dtype, void* stream) {
    if (dtype != MWC_F32 && dtype != MWC_F16 && dtype != MWC_BF16)
        return ex_fail(MWC_ERR_INVALID, "u must be float32/float16/bfloat16 (dtype code %d)", dtype);
    if (z != nullptr && (out == nullptr || out_z == nullptr))
        return ex_fail(MWC_ERR_INVALID, "with z, both out (ungated) and out_z are required");
    if (!delta) return ex_fail(MWC_ERR_INVALID, "u, delta, A, B_ssm, C_ssm and D_ssm are required");
    if (B < 0 || L < 0 || D < 0) return ex_fail(MWC_ERR_INVALID, "negative size");
    const int64_t n = B * L * D;
    const int64_t es = dtype == MWC_F32 ? 4 : 2;
    const bool transform = delta_bias != nullptr || delta_softplus != 0;
    const int64_t head = transform ? ex_align(n * es) : 0;
    if (transform && (workspace == nullptr || workspace_bytes < head))
        return ex_fail(MWC_ERR_WORKSPACE, "extended forward workspace of at least %lld bytes required",
                            (long long)mwc_ss_fwd_ex_workspace_bytes(B, L, D, dtype));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const void* dl = delta;
    if (transform && n > 0) {
        cudaError_t e = MWC_EX_DISPATCH(launch_delta_eff, dtype, delta, delta_bias, delta_softplus, workspace, n, D, s);
        if (e != cudaSuccess) return ex_fail(MWC_ERR_CUDA, "delta transform launch: %s", cudaGetErrorString(e));
        dl = workspace;
    }
    char* ws = static_cast<char*>(workspace);
    int rc = mwc_ss_fwd(u, dl, A, Bm, Cm, Dv, h_prev, out, h_last, ckpt, nullptr,
                        ws ? ws + head : nullptr, ws ? workspace_bytes - head : 0, B, L, D, dtype, stream);
    if (rc != MWC_OK) return rc;
    if (z != nullptr && n > 0) {
        cudaError_t e = MWC_EX_DISPATCH(launch_gate_fwd, dtype, out, z, out_z, n, s);
        if (e != cudaSuccess) return ex_fail(MWC_ERR_CUDA, "gate launch: %s", cudaGetErrorString(e));
    }
    return report_ok();
}

int64_t mwc_ss_bwd_ex_workspace_bytes(int64_t B, int64_t L, int64_t D, int dtype) {
    if (B <= 0 || L <= 0 || D <= 0) return 0;
    const int64_t es = dtype == MWC_F32 ? 4 : 2;
    const int64_t nchunk = (B * L + EX_ROWS_PER_CHUNK - 1) / EX_ROWS_PER_CHUNK;
    return 2 * ex_align(B * L * D * es) + ex_align(nchunk * D * 4) + mwc_ss_bwd_workspace_bytes(B, L, D, dtype);
}

int mwc_ss_bwd_ex(const void* u, const void* delta, const void* A, const void* Bm, const void* Cm,
                  const void* Dv, const void* z, const void* delta_bias, int delta_softplus,
                  const void* h_prev, const void* out, const void* dout, const void* dh_last,
                  const float* ckpt, void* du, void* ddelta, void* dA, void* dB, void* dC, void* dD,
                  void* ddelta_bias, void* dz, void* dh_prev, void* workspace, int64_t workspace_bytes,
                  int64_t B, int64_t L, int64_t D, int dtype, void* stream) {
    if (dtype != MWC_F32 && dtype != MWC_F16 && dtype != MWC_BF16)
        return ex_fail(MWC_ERR_INVALID, "u must be float32/float16/bfloat16 (dtype code %d)", dtype);
    if (z != nullptr && (out == nullptr || dz == nullptr))
        return ex_fail(MWC_ERR_INVALID, "with z, the ungated forward output and dz are required");
    if (!delta || !dout || !ddelta) return ex_fail(MWC_ERR_INVALID, "delta, dout and ddelta are required");
    if (B < 0 || L < 0 || D < 0) return ex_fail(MWC_ERR_INVALID, "negative size");
    const int64_t n = B * L * D, rows = B * L;
    const int64_t es = dtype == MWC_F32 ? 4 : 2;
    const int64_t nchunk = (rows + EX_ROWS_PER_CHUNK - 1) / EX_ROWS_PER_CHUNK;
    const int64_t big = ex_align(n * es);
    const int64_t head = 2 * big + ex_align(nchunk * D * 4);
    if (n > 0 && (workspace == nullptr || workspace_bytes < head))
        return ex_fail(MWC_ERR_WORKSPACE, "extended backward workspace of at least %lld bytes required",
                            (long long)mwc_ss_bwd_ex_workspace_bytes(B, L, D, dtype));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    char* ws = static_cast<char*>(workspace);
    const bool transform = delta_bias != nullptr || delta_softplus != 0;
    const void* dl = delta;
    const void* g = dout;
    if (n > 0 && transform) {
        cudaError_t e = MWC_EX_DISPATCH(launch_delta_eff, dtype, delta, delta_bias, delta_softplus, ws, n, D, s);
        if (e != cudaSuccess) return ex_fail(MWC_ERR_CUDA, "delta transform launch: %s", cudaGetErrorString(e));
        dl = ws;
    }
    if (n > 0 && z != nullptr) {
        cudaError_t e = MWC_EX_DISPATCH(launch_gate_bwd, dtype, dout, z, out, ws + big, dz, n, s);
        if (e != cudaSuccess) return ex_fail(MWC_ERR_CUDA, "gate backward launch: %s", cudaGetErrorString(e));
        g = ws + big;
    }
    int rc = mwc_ss_bwd(u, dl, A, Bm, Cm, Dv, h_prev, g, dh_last, ckpt, du, ddelta, dA, dB, dC, dD, dh_prev,
                        ws ? ws + head : nullptr, ws ? workspace_bytes - head : 0, B, L, D, dtype, stream);
    if (rc != MWC_OK) return rc;
    if (n > 0 && (delta_softplus != 0 || ddelta_bias != nullptr)) {
        float* partial = ddelta_bias != nullptr ? reinterpret_cast<float*>(ws + 2 * big) : nullptr;
        cudaError_t e = MWC_EX_DISPATCH(launch_ddelta, dtype, ddelta, delta, delta_bias, delta_softplus, partial,
                                        rows, D, ddelta_bias, s);
        if (e != cudaSuccess) return ex_fail(MWC_ERR_CUDA, "delta backward launch: %s", cudaGetErrorString(e));
    }
    return report_ok();
}

}  // extern "C"
