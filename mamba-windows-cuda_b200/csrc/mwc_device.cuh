// Device-side helpers shared by the selective-scan and linear-scan kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace mwc {

constexpr int NSTATE = 16;   // N: states per channel (the reference supports only 16)
constexpr int CK = 16;       // checkpoint / backward recompute chunk, in time steps
constexpr int DPRE_LT = 32;  // time steps per delta-prefix record (the persistent forward's tile)
constexpr int FX_CHUNK_TILES = 8;   // records per chunk of the chunked sequence-sharding fixup
constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;
// safe_exp in the reference clamps the natural exponent to [-88, 88]; in base 2 the
// upper bound is 88 * log2(e). (The lower clamp needs no code: ex2.approx.ftz already
// returns 0 below 2^-126, as the clamped __expf(-88) flushes to 0 under fast math.)
constexpr float ARG2_HI = 88.0f * 1.4426950408889634f;
constexpr unsigned FULL = 0xffffffffu;

// 2^x on the MUFU pipe (ex2.approx.ftz.f32: max rel. error 2^-22, subnormals flushed).
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

template <typename T> __device__ __forceinline__ T zero_v();
template <> __device__ __forceinline__ float zero_v<float>() { return 0.f; }
template <> __device__ __forceinline__ __half zero_v<__half>() { return __float2half_rn(0.f); }
template <> __device__ __forceinline__ __nv_bfloat16 zero_v<__nv_bfloat16>() { return __float2bfloat16_rn(0.f); }

// Copy a ROWS x COLS tile of a row-major matrix (row stride ld elements) into shared
// memory, zero-filling rows >= nrows and columns >= ncols. When `vec` holds (uniform per
// CTA: base, ld and col0 16-byte aligned and the tile fully in range), 16-byte vector
// loads are used; otherwise element loads. All NT threads participate.
template <typename T, int ROWS, int COLS, int NT>
__device__ __forceinline__ void load_tile(T (*dst)[COLS], const T* __restrict__ src,
                                          int64_t ld, int nrows, int ncols, bool vec) {
    constexpr int VEC = 16 / sizeof(T);
    if constexpr (COLS % VEC == 0) {
        if (vec && nrows == ROWS && ncols == COLS) {
            constexpr int CV = COLS / VEC;
            for (int idx = threadIdx.x; idx < ROWS * CV; idx += NT) {
                int r = idx / CV, c = (idx % CV) * VEC;
                *reinterpret_cast<uint4*>(&dst[r][c]) =
                    __ldg(reinterpret_cast<const uint4*>(src + r * ld + c));
            }
            return;
        }
    }
    for (int idx = threadIdx.x; idx < ROWS * COLS; idx += NT) {
        int r = idx / COLS, c = idx % COLS;
        T v = zero_v<T>();
        if (r < nrows && c < ncols) v = src[r * ld + c];
        dst[r][c] = v;
    }
}

// Same as load_tile but converts to float (used for the small B/C rows).
template <typename T, int ROWS, int COLS, int NT>
__device__ __forceinline__ void load_tile_f32(float (*dst)[COLS], const T* __restrict__ src,
                                              int64_t ld, int nrows) {
    for (int idx = threadIdx.x; idx < ROWS * COLS; idx += NT) {
        int r = idx / COLS, c = idx % COLS;
        dst[r][c] = (r < nrows) ? to_f(src[r * ld + c]) : 0.f;
    }
}

// Store a ROWS x COLS shared tile to global memory, rows < nrows and columns < ncols only.
template <typename T, int ROWS, int COLS, int NT>
__device__ __forceinline__ void store_tile(T* __restrict__ dst, const T (*src)[COLS],
                                           int64_t ld, int nrows, int ncols, bool vec) {
    constexpr int VEC = 16 / sizeof(T);
    if constexpr (COLS % VEC == 0) {
        if (vec && nrows == ROWS && ncols == COLS) {
            constexpr int CV = COLS / VEC;
            for (int idx = threadIdx.x; idx < ROWS * CV; idx += NT) {
                int r = idx / CV, c = (idx % CV) * VEC;
                *reinterpret_cast<uint4*>(dst + r * ld + c) =
                    *reinterpret_cast<const uint4*>(&src[r][c]);
            }
            return;
        }
    }
    for (int idx = threadIdx.x; idx < ROWS * COLS; idx += NT) {
        int r = idx / COLS, c = idx % COLS;
        if (r < nrows && c < ncols) dst[r * ld + c] = src[r][c];
    }
}

}  // namespace mwc
