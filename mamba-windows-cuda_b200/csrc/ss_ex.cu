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

// softplus and the logistic function through the fast exp / log / divide intrinsics: these
// kernels stream 4-10 bytes per element, and the precise log1pf / expf / IEEE division made
// them compute-bound. Errors: softplus a few 1e-7 absolute (the log of 1 + e^x near 1),
// sigmoid a few ulp; sigmoid is 0 below x = -87 and softplus is x above 20.
__device__ __forceinline__ float softplus_f(float x) { return x <= 20.f ? __logf(1.f + __expf(x)) : x; }
__device__ __forceinline__ float sigmoid_f(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }

constexpr int EX_THREADS = 256;
constexpr int EX_ROWS_PER_CHUNK = 64;    // rows of B*L summed per dbias partial

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

// dbias[d] = sum over chunks of partial[chunk][d]. Block = 32 channels x 8 lanes: lane j
// sums chunks j, j + 8, ... in order, then the 8 sums are added in lane order (fixed order,
// so the result is reproducible).
constexpr int EX_FINAL_SPLIT = 8;
template <typename T>
__global__ void dbias_final_kernel(const float* __restrict__ partial, int64_t nchunk, int64_t D, T* __restrict__ dbias) {
    __shared__ float part[EX_FINAL_SPLIT][32];
    const int c = threadIdx.x & 31, j = threadIdx.x >> 5;
    const int64_t d = (int64_t)blockIdx.x * 32 + c;
    float sum = 0.f;
    if (d < D)
        for (int64_t k = j; k < nchunk; k += EX_FINAL_SPLIT) sum += partial[k * D + d];
    part[j][c] = sum;
    __syncthreads();
    if (j == 0 && d < D) {
        float t = part[0][c];
#pragma unroll
        for (int q = 1; q < EX_FINAL_SPLIT; ++q) t += part[q][c];
        dbias[d] = from_f<T>(t);
    }
}

// ---- 16-byte vector forms (8 half / bf16 or 4 float elements per thread step) ----
template <typename T>
struct VecT {
    static constexpr int N = 16 / (int)sizeof(T);
};

template <typename T>
__device__ __forceinline__ void ld_vec(const T* p, float (&v)[VecT<T>::N]) {
    const uint4 raw = *reinterpret_cast<const uint4*>(p);
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int k = 0; k < VecT<T>::N; ++k) v[k] = to_f(e[k]);
}

template <typename T>
__device__ __forceinline__ void st_vec(T* p, const float (&v)[VecT<T>::N]) {
    uint4 raw;
    T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int k = 0; k < VecT<T>::N; ++k) e[k] = from_f<T>(v[k]);
    *reinterpret_cast<uint4*>(p) = raw;
}

template <typename T>
__global__ void delta_eff_vec_kernel(const T* __restrict__ delta, const T* __restrict__ bias, int softplus,
                                     T* __restrict__ out, int64_t nv, int64_t D) {
    constexpr int N = VecT<T>::N;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    // channel of the vector, advanced by the grid stride without a division per step
    const int64_t cstep = (stride * N) % D;
    int64_t col = (i0 * N) % D;
    for (int64_t i = i0; i < nv; i += stride) {
        float v[N], b[N];
        ld_vec<T>(delta + i * N, v);
        if (bias != nullptr) ld_vec<T>(bias + col, b);
        col += cstep;
        if (col >= D) col -= D;
#pragma unroll
        for (int k = 0; k < N; ++k) {
            const float x = v[k] + (bias != nullptr ? b[k] : 0.f);
            v[k] = softplus ? softplus_f(x) : x;
        }
        st_vec<T>(out + i * N, v);
    }
}

template <typename T>
__global__ void gate_fwd_vec_kernel(const T* __restrict__ y, const T* __restrict__ z, T* __restrict__ out_z,
                                    int64_t nv) {
    constexpr int N = VecT<T>::N;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
        float yv[N], zv[N];
        ld_vec<T>(y + i * N, yv);
        ld_vec<T>(z + i * N, zv);
#pragma unroll
        for (int k = 0; k < N; ++k) yv[k] = yv[k] * zv[k] * sigmoid_f(zv[k]);
        st_vec<T>(out_z + i * N, yv);
    }
}

template <typename T>
__global__ void gate_bwd_vec_kernel(const T* __restrict__ dout, const T* __restrict__ z, const T* __restrict__ y,
                                    T* __restrict__ gy, T* __restrict__ dz, int64_t nv) {
    constexpr int N = VecT<T>::N;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
        float g[N], zv[N], yv[N], a[N], b[N];
        ld_vec<T>(dout + i * N, g);
        ld_vec<T>(z + i * N, zv);
        ld_vec<T>(y + i * N, yv);
#pragma unroll
        for (int k = 0; k < N; ++k) {
            const float sg = sigmoid_f(zv[k]);
            a[k] = g[k] * zv[k] * sg;
            b[k] = g[k] * yv[k] * sg * (1.f + zv[k] * (1.f - sg));
        }
        st_vec<T>(gy + i * N, a);
        st_vec<T>(dz + i * N, b);
    }
}

// thread = one 16-byte group of channels for a chunk of rows (rows in order)
template <typename T>
__global__ void ddelta_vec_kernel(T* __restrict__ ddelta, const T* __restrict__ delta, const T* __restrict__ bias,
                                  int softplus, float* __restrict__ partial, int64_t rows, int64_t D) {
    constexpr int N = VecT<T>::N;
    const int64_t dv = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (dv * N >= D) return;
    const int64_t d0 = dv * N;
    const int64_t chunk = blockIdx.y;
    float bd[N];
    if (bias != nullptr) ld_vec<T>(bias + d0, bd);
    else {
#pragma unroll
        for (int k = 0; k < N; ++k) bd[k] = 0.f;
    }
    const int64_t r0 = chunk * EX_ROWS_PER_CHUNK;
    const int64_t r1 = rows < r0 + EX_ROWS_PER_CHUNK ? rows : r0 + EX_ROWS_PER_CHUNK;
    float acc[N];
#pragma unroll
    for (int k = 0; k < N; ++k) acc[k] = 0.f;
#pragma unroll 4
    for (int64_t r = r0; r < r1; ++r) {
        float g[N];
        ld_vec<T>(ddelta + r * D + d0, g);
        if (softplus) {
            float x[N];
            ld_vec<T>(delta + r * D + d0, x);
#pragma unroll
            for (int k = 0; k < N; ++k) g[k] *= sigmoid_f(x[k] + bd[k]);
            st_vec<T>(ddelta + r * D + d0, g);
        }
#pragma unroll
        for (int k = 0; k < N; ++k) acc[k] += g[k];
    }
    if (partial != nullptr) {
#pragma unroll
        for (int k = 0; k < N; ++k) partial[chunk * D + d0 + k] = acc[k];
    }
}

template <typename T>
static cudaError_t launch_delta_eff(const void* delta, const void* bias, int softplus, void* out, int64_t n,
                                    int64_t D, cudaStream_t s) {
    constexpr int N = VecT<T>::N;
    if (D % N == 0) {
        delta_eff_vec_kernel<T><<<ex_blocks(n / N), EX_THREADS, 0, s>>>(
            static_cast<const T*>(delta), static_cast<const T*>(bias), softplus, static_cast<T*>(out), n / N, D);
    } else {
        delta_eff_kernel<T><<<ex_blocks(n), EX_THREADS, 0, s>>>(static_cast<const T*>(delta), static_cast<const T*>(bias),
                                                                softplus, static_cast<T*>(out), n, D);
    }
    return cudaGetLastError();
}
template <typename T>
static cudaError_t launch_gate_fwd(const void* y, const void* z, void* out_z, int64_t n, cudaStream_t s) {
    constexpr int N = VecT<T>::N;
    if (n % N == 0) {
        gate_fwd_vec_kernel<T><<<ex_blocks(n / N), EX_THREADS, 0, s>>>(
            static_cast<const T*>(y), static_cast<const T*>(z), static_cast<T*>(out_z), n / N);
    } else {
        gate_fwd_kernel<T><<<ex_blocks(n), EX_THREADS, 0, s>>>(static_cast<const T*>(y), static_cast<const T*>(z),
                                                               static_cast<T*>(out_z), n);
    }
    return cudaGetLastError();
}
template <typename T>
static cudaError_t launch_gate_bwd(const void* dout, const void* z, const void* y, void* gy, void* dz, int64_t n,
                                   cudaStream_t s) {
    constexpr int N = VecT<T>::N;
    if (n % N == 0) {
        gate_bwd_vec_kernel<T><<<ex_blocks(n / N), EX_THREADS, 0, s>>>(
            static_cast<const T*>(dout), static_cast<const T*>(z), static_cast<const T*>(y), static_cast<T*>(gy),
            static_cast<T*>(dz), n / N);
    } else {
        gate_bwd_kernel<T><<<ex_blocks(n), EX_THREADS, 0, s>>>(static_cast<const T*>(dout), static_cast<const T*>(z),
                                                               static_cast<const T*>(y), static_cast<T*>(gy),
                                                               static_cast<T*>(dz), n);
    }
    return cudaGetLastError();
}
template <typename T>
static cudaError_t launch_ddelta(void* ddelta, const void* delta, const void* bias, int softplus, float* partial,
                                 int64_t rows, int64_t D, void* dbias, cudaStream_t s) {
    const int64_t nchunk = (rows + EX_ROWS_PER_CHUNK - 1) / EX_ROWS_PER_CHUNK;
    constexpr int N = VecT<T>::N;
    if (D % N == 0) {
        const int64_t groups = D / N;
        const int tpb = (int)std::min<int64_t>(EX_THREADS, ((groups + 31) / 32) * 32);
        dim3 grid((unsigned)((groups + tpb - 1) / tpb), (unsigned)nchunk);
        ddelta_vec_kernel<T><<<grid, tpb, 0, s>>>(static_cast<T*>(ddelta), static_cast<const T*>(delta),
                                                  static_cast<const T*>(bias), softplus, partial, rows, D);
    } else {
        dim3 grid((unsigned)((D + EX_THREADS - 1) / EX_THREADS), (unsigned)nchunk);
        ddelta_kernel<T><<<grid, EX_THREADS, 0, s>>>(static_cast<T*>(ddelta), static_cast<const T*>(delta),
                                                     static_cast<const T*>(bias), softplus, partial, rows, D);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || dbias == nullptr) return e;
    dbias_final_kernel<T><<<(unsigned)((D + 31) / 32), 32 * EX_FINAL_SPLIT, 0, s>>>(partial, nchunk, D,
                                                                                   static_cast<T*>(dbias));
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
