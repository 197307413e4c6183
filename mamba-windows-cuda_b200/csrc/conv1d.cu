// Causal depthwise conv1d, the producer of the scan's input u in Mamba's block (not in the
// reference; the official Mamba stack ships it as causal_conv1d). Channel-last layout like
// the scan:
//   x (B, L, D), weight (D, W) with W <= 4, bias (D) or NULL, x_prev (B, W-1, D) or NULL
//   (the W-1 inputs before t = 0, zero when NULL), activation 0 = none, 1 = SiLU:
//   pre[b,t,d] = bias[d] + sum_k weight[d,k] * x[b, t-(W-1)+k, d];   y = act(pre)
// Backward (dy given): dpre = dy * act'(pre) (pre recomputed from x);
//   dx[t] = sum_k weight[k] dpre[t+(W-1)-k],  dweight[k] = sum_{b,t} dpre[t] x[t-(W-1)+k],
//   dbias = sum_{b,t} dpre[t],  dx_prev[j] = sum_{k <= j} weight[k] dpre[j-k].
//
// HBM-bound. Two paths:
// * TMA-staged (rows of D * elem a multiple of 16 bytes, 16-byte aligned buffers): CTAs own a
//   256-byte channel block and stream (batch row, 64-step tile) items with their halo rows
//   through a shared-memory ring fed by a producer warp (conv1d_fwd_tma_kernel /
//   conv1d_bwd_tma_kernel below); dweight / dbias accumulate per CTA and are summed over a
//   shape-determined number of CTA partials in a fixed order.
// * Plain loads (any other row): a thread owns one channel group and a run of CV_RUN time
//   steps, keeps the last W-1 inputs (and, backward, the last W-1 dpre) in registers;
//   dweight / dbias partials per (b, run), then a fixed-order sum.
// Per element both paths do the same operations, so y and dx agree bitwise.
#include "mwc_b200.h"
#include "mwc_device.cuh"
#include "mwc_internal.h"
#include "mwc_tma.cuh"

#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <type_traits>

namespace mwc {

constexpr int CV_RUN = 64;   // time steps per thread
constexpr int CV_THREADS = 128;

template <typename T, int VEC>
__device__ __forceinline__ void cv_load(const T* p, float (&v)[VEC]) {
    if constexpr (VEC * sizeof(T) == 16) {
        const uint4 raw = *reinterpret_cast<const uint4*>(p);
        const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
        for (int k = 0; k < VEC; ++k) v[k] = to_f(e[k]);
    } else {
#pragma unroll
        for (int k = 0; k < VEC; ++k) v[k] = to_f(p[k]);
    }
}

template <typename T, int VEC>
__device__ __forceinline__ void cv_store(T* p, const float (&v)[VEC]) {
    if constexpr (VEC * sizeof(T) == 16) {
        uint4 raw;
        T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
        for (int k = 0; k < VEC; ++k) e[k] = from_f<T>(v[k]);
        *reinterpret_cast<uint4*>(p) = raw;
    } else {
#pragma unroll
        for (int k = 0; k < VEC; ++k) p[k] = from_f<T>(v[k]);
    }
}

// logistic function: one exponential and one fast reciprocal-multiply (error a few ulp; the
// result is 0 once exp(-x) passes 2^126, i.e. x < -87, where the true value is below 1e-38)
__device__ __forceinline__ float cv_sigmoid(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }

// s[q] = init[q] + sum_kk a[kk][q] * b[kk][q], accumulated in kk order. Channel pairs go
// through one packed fma.rn.f32x2; each of its lanes rounds like fmaf, so the result is
// bitwise the scalar chain (the element path, with one channel per thread, runs that chain).
template <int W, int V>
__device__ __forceinline__ void cv_taps(const float (&a)[W][V], const float (&b)[W][V], const float (&init)[V],
                                        float (&s)[V]) {
    if constexpr (V % 2 == 0) {
#pragma unroll
        for (int q = 0; q < V; q += 2) {
            float2 acc = make_float2(init[q], init[q + 1]);
#pragma unroll
            for (int kk = 0; kk < W; ++kk)
                acc = __ffma2_rn(make_float2(a[kk][q], a[kk][q + 1]), make_float2(b[kk][q], b[kk][q + 1]), acc);
            s[q] = acc.x;
            s[q + 1] = acc.y;
        }
    } else {
#pragma unroll
        for (int q = 0; q < V; ++q) {
            float acc = init[q];
#pragma unroll
            for (int kk = 0; kk < W; ++kk) acc = fmaf(a[kk][q], b[kk][q], acc);
            s[q] = acc;
        }
    }
}

// acc[kk][q] += x[q] * y[kk][q] for every tap (packed by channel pairs, like cv_taps)
template <int W, int V>
__device__ __forceinline__ void cv_accum(float (&acc)[W][V], const float (&x)[V], const float (&y)[W][V]) {
#pragma unroll
    for (int kk = 0; kk < W; ++kk) {
        if constexpr (V % 2 == 0) {
#pragma unroll
            for (int q = 0; q < V; q += 2) {
                const float2 r = __ffma2_rn(make_float2(x[q], x[q + 1]), make_float2(y[kk][q], y[kk][q + 1]),
                                            make_float2(acc[kk][q], acc[kk][q + 1]));
                acc[kk][q] = r.x;
                acc[kk][q + 1] = r.y;
            }
        } else {
#pragma unroll
            for (int q = 0; q < V; ++q) acc[kk][q] = fmaf(x[q], y[kk][q], acc[kk][q]);
        }
    }
}

// x at time t (t may be negative: from x_prev, or zero)
template <typename T, int VEC, int W>
__device__ __forceinline__ void cv_x_at(const T* x, const T* x_prev, int64_t b, int64_t t, int64_t L, int64_t D,
                                        int64_t d0, float (&v)[VEC]) {
    if (t >= 0) {
        cv_load<T, VEC>(x + (b * L + t) * D + d0, v);
    } else if (x_prev != nullptr) {
        cv_load<T, VEC>(x_prev + (b * (W - 1) + (t + (W - 1))) * D + d0, v);
    } else {
#pragma unroll
        for (int k = 0; k < VEC; ++k) v[k] = 0.f;
    }
}

template <typename T, int VEC, int W>
__global__ void __launch_bounds__(CV_THREADS) conv1d_fwd_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                                const T* __restrict__ bias, const T* __restrict__ x_prev,
                                                                int act, T* __restrict__ y, int64_t L, int64_t D) {
    const int64_t d0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * VEC;
    if (d0 >= D) return;
    const int64_t b = blockIdx.z;
    const int64_t t0 = (int64_t)blockIdx.y * CV_RUN;
    const int64_t t1 = t0 + CV_RUN < L ? t0 + CV_RUN : L;
    float wk[W][VEC], bv[VEC], win[W][VEC];
#pragma unroll
    for (int c = 0; c < VEC; ++c) {
#pragma unroll
        for (int k = 0; k < W; ++k) wk[k][c] = to_f(w[(d0 + c) * W + k]);
        bv[c] = bias != nullptr ? to_f(bias[d0 + c]) : 0.f;
    }
#pragma unroll
    for (int k = 0; k < W - 1; ++k) cv_x_at<T, VEC, W>(x, x_prev, b, t0 - (W - 1) + k, L, D, d0, win[k]);
    for (int64_t t = t0; t < t1; ++t) {
        cv_load<T, VEC>(x + (b * L + t) * D + d0, win[W - 1]);
        float o[VEC];
        cv_taps<W, VEC>(wk, win, bv, o);
        if (act) {
#pragma unroll
            for (int c = 0; c < VEC; ++c) o[c] = o[c] * cv_sigmoid(o[c]);
        }
        cv_store<T, VEC>(y + (b * L + t) * D + d0, o);
#pragma unroll
        for (int k = 0; k < W - 1; ++k)
#pragma unroll
            for (int c = 0; c < VEC; ++c) win[k][c] = win[k + 1][c];
    }
}

// dpre at time s (zero outside [0, L)); xw holds x[s-(W-1) .. s]
template <int VEC, int W>
__device__ __forceinline__ void cv_dpre(const float (&wk)[W][VEC], const float (&bv)[VEC], const float (&xw)[W][VEC],
                                        const float (&g)[VEC], int act, float (&dp)[VEC]) {
#pragma unroll
    for (int c = 0; c < VEC; ++c) dp[c] = g[c];
    if (act) {
        float pre[VEC];
        cv_taps<W, VEC>(wk, xw, bv, pre);
#pragma unroll
        for (int c = 0; c < VEC; ++c) {
            const float sg = cv_sigmoid(pre[c]);
            dp[c] = g[c] * sg * (1.f + pre[c] * (1.f - sg));
        }
    }
}

// Thread = (channel group, run of CV_RUN steps, batch row). Walks s over the run plus a
// look-ahead of W-1 steps (the dpre that dx of the run's last steps needs), emitting
// dx[s-(W-1)] once dpre[s-(W-1) .. s] are known; dweight / dbias partials over the run's own s.
template <typename T, int VEC, int W>
__global__ void __launch_bounds__(CV_THREADS) conv1d_bwd_kernel(
    const T* __restrict__ x, const T* __restrict__ w, const T* __restrict__ bias, const T* __restrict__ x_prev,
    int act, const T* __restrict__ dy, T* __restrict__ dx, T* __restrict__ dx_prev, float* __restrict__ part,
    int64_t L, int64_t D, int64_t nrun) {
    const int64_t d0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * VEC;
    if (d0 >= D) return;
    const int64_t b = blockIdx.z;
    const int64_t run = blockIdx.y;
    const int64_t t0 = run * CV_RUN;
    const int64_t t1 = t0 + CV_RUN < L ? t0 + CV_RUN : L;
    float wk[W][VEC], bv[VEC], xw[W][VEC], dq[W][VEC];   // dq[k] = dpre[s - (W-1) + k]
    float aw[W][VEC], ab[VEC];
#pragma unroll
    for (int c = 0; c < VEC; ++c) {
#pragma unroll
        for (int k = 0; k < W; ++k) {
            wk[k][c] = to_f(w[(d0 + c) * W + k]);
            aw[k][c] = 0.f;
            dq[k][c] = 0.f;
        }
        bv[c] = bias != nullptr ? to_f(bias[d0 + c]) : 0.f;
        ab[c] = 0.f;
    }
#pragma unroll
    for (int k = 0; k < W - 1; ++k) cv_x_at<T, VEC, W>(x, x_prev, b, t0 - (W - 1) + k, L, D, d0, xw[k]);
    const int64_t send = t1 + (W - 1) < L ? t1 + (W - 1) : L;   // last s with a dpre, + 1
    for (int64_t s = t0; s < t1 + (W - 1); ++s) {
        float dp[VEC];
        if (s < send) {
            float g[VEC];
            cv_load<T, VEC>(x + (b * L + s) * D + d0, xw[W - 1]);
            cv_load<T, VEC>(dy + (b * L + s) * D + d0, g);
            cv_dpre<VEC, W>(wk, bv, xw, g, act, dp);
            if (s < t1) {
#pragma unroll
                for (int c = 0; c < VEC; ++c) ab[c] += dp[c];
                cv_accum<W, VEC>(aw, dp, xw);
            }
        } else {
#pragma unroll
            for (int c = 0; c < VEC; ++c) dp[c] = 0.f;
        }
        // slide: dq holds dpre[s-(W-1) .. s]
#pragma unroll
        for (int k = 0; k < W - 1; ++k)
#pragma unroll
            for (int c = 0; c < VEC; ++c) dq[k][c] = dq[k + 1][c];
#pragma unroll
        for (int c = 0; c < VEC; ++c) dq[W - 1][c] = dp[c];
        // dx[t] for t = s - (W-1): sum_k w[k] dpre[t + (W-1) - k] = sum_k w[k] dq[W-1-k]
        const int64_t t = s - (W - 1);
        if (t >= t0 || (run == 0 && dx_prev != nullptr && t >= -(W - 1))) {
            float o[VEC];
#pragma unroll
            for (int c = 0; c < VEC; ++c) {
                float a = 0.f;
#pragma unroll
                for (int k = 0; k < W; ++k) a = fmaf(wk[k][c], dq[W - 1 - k][c], a);
                o[c] = a;
            }
            if (t >= t0) cv_store<T, VEC>(dx + (b * L + t) * D + d0, o);
            else cv_store<T, VEC>(dx_prev + (b * (W - 1) + (t + (W - 1))) * D + d0, o);
        }
        if (s < send) {
#pragma unroll
            for (int k = 0; k < W - 1; ++k)
#pragma unroll
                for (int c = 0; c < VEC; ++c) xw[k][c] = xw[k + 1][c];
        }
    }
    // partials: part[(b * nrun + run)][W + 1][D] (W weight taps, then the bias)
    float* pp = part + (b * nrun + run) * (W + 1) * D;
#pragma unroll
    for (int c = 0; c < VEC; ++c) {
#pragma unroll
        for (int k = 0; k < W; ++k) pp[k * D + d0 + c] = aw[k][c];
        pp[W * D + d0 + c] = ab[c];
    }
}

// dweight[d, k] and dbias[d]: sums of the partials over (b, run) in that order.
template <typename T, int W>
__global__ void conv1d_reduce_kernel(const float* __restrict__ part, int64_t nparts, int64_t D,
                                     T* __restrict__ dw, T* __restrict__ db) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)(W + 1) * D) return;
    const int64_t k = idx / D, d = idx % D;
    float s = 0.f;
    for (int64_t p = 0; p < nparts; ++p) s += part[(p * (W + 1) + k) * D + d];
    if (k < W) dw[d * W + k] = from_f<T>(s);
    else if (db != nullptr) db[d] = from_f<T>(s);
}

// ------------------------------------------------------------------ TMA-staged kernels
// A CTA owns one channel block (CT_ROWB bytes of a row: 128 16-bit or 64 float32 channels)
// and walks a fixed, strided list of (batch row, CT_TT-step tile) items. A producer warp
// streams each tile with its halo rows into a shared-memory ring through TMA, so the bytes in
// flight per SM are bounded by shared memory, not by registers; 256 compute threads own 4
// channels x R rows of a tile each (R = 8 for 16-bit types, 4 for float32). Tiles reload
// their own halo (L2 hits: the neighbouring tile is read at about the same time).
constexpr int CT_ROWB = 256;      // bytes of one tile row (the channel block)
constexpr int CT_TT = 64;         // time steps per tile
constexpr int CT_THREADS = 256;   // compute threads (8 warps); one producer warp on top
constexpr int CT_FWD_CPT = 4;     // channels per compute thread, forward
constexpr int CT_BWD_CPT = 2;     // and backward (half the registers: 2 CTAs per SM)
constexpr int CT_HALO = 3;        // halo rows before a tile (and, backward, after it): W - 1 <= 3
constexpr int CT_FWD_ST = 4;      // forward ring: 4 stages of 17 KB, 3 CTAs per SM
constexpr int CT_FWD_CTAS_PER_SM = 3;
constexpr int CT_BWD_ST = 2;      // backward ring: 2 stages of 35 KB plus the exchange, 2 CTAs per SM
// Backward CTA budget (2 per SM of a 148-SM part). It fixes the number of dweight / dbias
// partials, and so their summation order, as a function of the shape alone.
constexpr int CT_BWD_CTAS = 296;

// Sticky bounded-wait error word of the TMA conv kernels (set once a wait gives up).
__device__ int g_cv_err;

__device__ __forceinline__ void cv_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Named barrier 1 over the compute threads; returns whether any of them passed true.
__device__ __forceinline__ bool cv_bar_any(bool v) {
    int r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.s32 q, %1, 0;\n\t"
        "bar.red.or.pred p, 1, %2, q;\n\t"
        "selp.s32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"((int)v), "n"(CT_THREADS)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ void cv_bar() { asm volatile("bar.sync 1, %0;" ::"n"(CT_THREADS) : "memory"); }

// N (2 or 4) consecutive channels from / to global or shared memory, as float
template <typename T>
__device__ __forceinline__ float2 ct_pair(uint32_t u) {
    if constexpr (std::is_same<T, __half>::value) return __half22float2(*reinterpret_cast<const __half2*>(&u));
    else return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u));
}
template <typename T>
__device__ __forceinline__ uint32_t ct_pack(float a, float b) {
    if constexpr (std::is_same<T, __half>::value) {
        __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    } else {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
}
template <typename T, int N>
__device__ __forceinline__ void ct_ld(const T* p, float (&v)[N]) {
    static_assert(N == 2 || N == 4, "2 or 4 channels");
    if constexpr (std::is_same<T, float>::value) {
        if constexpr (N == 4) {
            const float4 q = *reinterpret_cast<const float4*>(p);
            v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
        } else {
            const float2 q = *reinterpret_cast<const float2*>(p);
            v[0] = q.x; v[1] = q.y;
        }
    } else if constexpr (N == 4) {
        const uint2 q = *reinterpret_cast<const uint2*>(p);
        const float2 a = ct_pair<T>(q.x), b = ct_pair<T>(q.y);
        v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
    } else {
        const float2 a = ct_pair<T>(*reinterpret_cast<const uint32_t*>(p));
        v[0] = a.x; v[1] = a.y;
    }
}
template <typename T, int N>
__device__ __forceinline__ void ct_st(T* p, const float (&v)[N]) {
    if constexpr (std::is_same<T, float>::value) {
        if constexpr (N == 4) *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
        else *reinterpret_cast<float2*>(p) = make_float2(v[0], v[1]);
    } else if constexpr (N == 4) {
        *reinterpret_cast<uint2*>(p) = make_uint2(ct_pack<T>(v[0], v[1]), ct_pack<T>(v[2], v[3]));
    } else {
        *reinterpret_cast<uint32_t*>(p) = ct_pack<T>(v[0], v[1]);
    }
}

template <typename T, int P>
struct CtShape {
    static constexpr int CC = CT_ROWB / (int)sizeof(T);   // channels per block
    static constexpr int COLS = CC / P;                    // compute threads per tile row
    static constexpr int G = CT_THREADS / COLS;            // row groups
    static constexpr int R = CT_TT / G;                    // rows per compute thread
    static_assert(R >= CT_HALO, "a row group must cover the halo");
};

// Producer (one thread): item k of this CTA (j = seg + k * nseg) goes to stage k % NST; the x
// box at (c0, t0 - CT_HALO, b) and, with tm_g, the dy box at (c0, t0, b) right after it.
template <int NST>
__device__ __forceinline__ void cv_produce(const CUtensorMap* tm_x, const CUtensorMap* tm_g, unsigned char* smem,
                                           int stb, int xbytes, uint64_t* full, uint64_t* empty, int c0, int seg,
                                           int nseg, int nitems, int ntiles, int* err) {
    prefetch_tmap(tm_x);
    if (tm_g != nullptr) prefetch_tmap(tm_g);
    int k = 0;
    for (int j = seg; j < nitems; j += nseg, ++k) {
        const int st = k % NST;
        if (k >= NST && !mbar_wait(&empty[st], ((k / NST) - 1) & 1, err)) break;
        const int b = j / ntiles, t0 = (j % ntiles) * CT_TT;
        unsigned char* dst = smem + st * stb;
        mbar_expect_tx(&full[st], (unsigned)stb);
        tma_load_3d(dst, tm_x, &full[st], c0, t0 - CT_HALO, b);
        if (tm_g != nullptr) tma_load_3d(dst + xbytes, tm_g, &full[st], c0, t0, b);
    }
    // copies possibly still in flight (consumers that stopped early): wait for them, bounded
    for (int q = k > NST ? k - NST : 0; q < k; ++q) mbar_wait(&full[q % NST], (q / NST) & 1, nullptr);
}

template <typename T, int W>
__global__ void __launch_bounds__(CT_THREADS + 32, CT_FWD_CTAS_PER_SM) conv1d_fwd_tma_kernel(
    const __grid_constant__ CUtensorMap tm_x, const T* __restrict__ w, const T* __restrict__ bias,
    const T* __restrict__ x_prev, int act, T* __restrict__ y, int B, int L, int D, int ncb, int nseg) {
    constexpr int P = CT_FWD_CPT;
    using S = CtShape<T, P>;
    constexpr int CC = S::CC, COLS = S::COLS, R = S::R, NST = CT_FWD_ST;
    constexpr int STB = (CT_TT + CT_HALO) * CT_ROWB;
    extern __shared__ __align__(128) unsigned char cv_smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(cv_smem + NST * STB);
    uint64_t* empty = full + NST;
    int* err = &g_cv_err;
    const int tid = threadIdx.x;
    const int cb = blockIdx.x % ncb, seg = blockIdx.x / ncb;
    const int ntiles = (L + CT_TT - 1) / CT_TT;
    const int nitems = B * ntiles;
    if (tid == 0) {
        for (int s = 0; s < NST; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], CT_THREADS / 32);
        }
        fence_mbar_init();
    }
    __syncthreads();
    if (tid >= CT_THREADS) {
        if (tid == CT_THREADS)
            cv_produce<NST>(&tm_x, nullptr, cv_smem, STB, STB, full, empty, cb * CC, seg, nseg, nitems, ntiles, err);
        return;
    }
    const int col = tid % COLS, rg = tid / COLS, lane = tid & 31;
    const int c = cb * CC + col * P;
    const bool valid = c < D;
    const int r0 = rg * R;
    float wk[W][P], bv[P];
#pragma unroll
    for (int q = 0; q < P; ++q) {
#pragma unroll
        for (int k = 0; k < W; ++k) wk[k][q] = valid ? to_f(w[(int64_t)(c + q) * W + k]) : 0.f;
        bv[q] = valid && bias != nullptr ? to_f(bias[c + q]) : 0.f;
    }
    int k = 0;
    for (int j = seg; j < nitems; j += nseg, ++k) {
        const int st = k % NST;
        if (!__all_sync(0xffffffffu, mbar_wait(&full[st], (k / NST) & 1, err))) break;
        const int b = j / ntiles, t0 = (j % ntiles) * CT_TT;
        const T* sx = reinterpret_cast<const T*>(cv_smem + st * STB) + col * P;   // row r: x[t0 - 3 + r]
        float win[W][P];
#pragma unroll
        for (int q = 0; q < W - 1; ++q) {
            const int t = t0 + r0 - (W - 1) + q;
            if (t < 0 && x_prev != nullptr) {
                if (valid) {
                    ct_ld<T, P>(x_prev + ((int64_t)b * (W - 1) + t + (W - 1)) * D + c, win[q]);
                } else {
#pragma unroll
                    for (int p = 0; p < P; ++p) win[q][p] = 0.f;
                }
            } else {
                ct_ld<T, P>(sx + (r0 + CT_HALO - (W - 1) + q) * CC, win[q]);
            }
        }
#pragma unroll
        for (int i = 0; i < R; ++i) {
            ct_ld<T, P>(sx + (r0 + CT_HALO + i) * CC, win[W - 1]);
            float o[P];
            cv_taps<W, P>(wk, win, bv, o);
            if (act) {
#pragma unroll
                for (int q = 0; q < P; ++q) o[q] = o[q] * cv_sigmoid(o[q]);
            }
            const int t = t0 + r0 + i;
            if (valid && t < L) ct_st<T, P>(y + ((int64_t)b * L + t) * D + c, o);
#pragma unroll
            for (int kk = 0; kk < W - 1; ++kk)
#pragma unroll
                for (int q = 0; q < P; ++q) win[kk][q] = win[kk + 1][q];
        }
        __syncwarp();
        if (lane == 0) cv_arrive(&empty[st]);
    }
}

// dx at the row whose dpre window is dq: sum_kk w[kk] dq[W-1-kk], stored when do_store
template <typename T, int W, int P>
__device__ __forceinline__ void cv_dx_emit(const float (&wk)[W][P], const float (&dq)[W][P], bool do_store,
                                           T* dst) {
    float o[P], rq[W][P];
    const float zero[P] = {};
#pragma unroll
    for (int kk = 0; kk < W; ++kk)
#pragma unroll
        for (int q = 0; q < P; ++q) rq[kk][q] = dq[W - 1 - kk][q];
    cv_taps<W, P>(wk, rq, zero, o);
    if (do_store) ct_st<T, P>(dst, o);
}

// Backward. Stage = x rows t0-3 .. t0+CT_TT+2 then dy rows t0 .. t0+CT_TT+2 (zero past L).
// A thread steps through its R rows computing dpre, the dweight / dbias sums and dx of the
// rows whose dpre window is complete; its first W-1 dpre go to a double-buffered exchange
// from which the row group above finishes dx of its last W-1 rows (the last row group
// computes the W-1 dpre after the tile itself).
template <typename T, int W>
__global__ void __launch_bounds__(CT_THREADS + 32, 2) conv1d_bwd_tma_kernel(
    const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_g, const T* __restrict__ w,
    const T* __restrict__ bias, const T* __restrict__ x_prev, int act, T* __restrict__ dx, T* __restrict__ dx_prev,
    float* __restrict__ part, int B, int L, int D, int ncb, int nseg) {
    constexpr int P = CT_BWD_CPT;
    using S = CtShape<T, P>;
    constexpr int CC = S::CC, COLS = S::COLS, G = S::G, R = S::R, NST = CT_BWD_ST;
    constexpr int XB = (CT_TT + 2 * CT_HALO) * CT_ROWB;
    constexpr int STB = XB + (CT_TT + CT_HALO) * CT_ROWB;
    constexpr int XCH = G * CT_HALO * CC;   // floats per exchange buffer
    static_assert(G * (W + 1) * CC * 4 <= NST * STB, "partial sums reuse the ring");
    extern __shared__ __align__(128) unsigned char cv_smem[];
    float* xch = reinterpret_cast<float*>(cv_smem + NST * STB);
    uint64_t* full = reinterpret_cast<uint64_t*>(xch + 2 * XCH);
    uint64_t* empty = full + NST;
    int* err = &g_cv_err;
    const int tid = threadIdx.x;
    const int cb = blockIdx.x % ncb, seg = blockIdx.x / ncb;
    const int ntiles = (L + CT_TT - 1) / CT_TT;
    const int nitems = B * ntiles;
    if (tid == 0) {
        for (int s = 0; s < NST; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], CT_THREADS / 32);
        }
        fence_mbar_init();
    }
    __syncthreads();
    if (tid >= CT_THREADS) {
        if (tid == CT_THREADS)
            cv_produce<NST>(&tm_x, &tm_g, cv_smem, STB, XB, full, empty, cb * CC, seg, nseg, nitems, ntiles, err);
        return;
    }
    const int col = tid % COLS, rg = tid / COLS, lane = tid & 31;
    const int c = cb * CC + col * P;
    const bool valid = c < D;
    const int r0 = rg * R;
    float wk[W][P], bv[P], aw[W][P], ab[P];
#pragma unroll
    for (int q = 0; q < P; ++q) {
#pragma unroll
        for (int k = 0; k < W; ++k) {
            wk[k][q] = valid ? to_f(w[(int64_t)(c + q) * W + k]) : 0.f;
            aw[k][q] = 0.f;
        }
        bv[q] = valid && bias != nullptr ? to_f(bias[c + q]) : 0.f;
        ab[q] = 0.f;
    }
    int k = 0;
    for (int j = seg; j < nitems; j += nseg, ++k) {
        const int st = k % NST;
        // a failed wait leaves the stage undefined; the barrier below turns it into a uniform exit
        const bool ok = mbar_wait(&full[st], (k / NST) & 1, err);
        const int b = j / ntiles, t0 = (j % ntiles) * CT_TT;
        const T* sx = reinterpret_cast<const T*>(cv_smem + st * STB) + col * P;        // row r: x[t0 - 3 + r]
        const T* sg = reinterpret_cast<const T*>(cv_smem + st * STB + XB) + col * P;   // row r: dy[t0 + r]
        float win[W][P];
#pragma unroll
        for (int q = 0; q < W - 1; ++q) {
            const int t = t0 + r0 - (W - 1) + q;
            if (t < 0 && x_prev != nullptr) {
                if (valid) {
                    ct_ld<T, P>(x_prev + ((int64_t)b * (W - 1) + t + (W - 1)) * D + c, win[q]);
                } else {
#pragma unroll
                    for (int p = 0; p < P; ++p) win[q][p] = 0.f;
                }
            } else {
                ct_ld<T, P>(sx + (r0 + CT_HALO - (W - 1) + q) * CC, win[q]);
            }
        }
        // dq[kk] = dpre[s - (W-1) + kk] while stepping s (zero before the thread's first row), so
        // dx[s - (W-1)] = sum_kk w[kk] dq[W-1-kk] is emitted as soon as dpre[s] is known
        float dq[W][P];
#pragma unroll
        for (int kk = 0; kk < W; ++kk)
#pragma unroll
            for (int q = 0; q < P; ++q) dq[kk][q] = 0.f;
        float* xb = xch + (k & 1) * XCH;
        const bool emit_prev = dx_prev != nullptr && t0 == 0 && rg == 0 && valid;
#pragma unroll
        for (int i = 0; i < R; ++i) {
            float g[P], dp[P];
            ct_ld<T, P>(sx + (r0 + CT_HALO + i) * CC, win[W - 1]);
            ct_ld<T, P>(sg + (r0 + i) * CC, g);
            cv_dpre<P, W>(wk, bv, win, g, act, dp);
#pragma unroll
            for (int q = 0; q < P; ++q) ab[q] += dp[q];
            cv_accum<W, P>(aw, dp, win);
            if (i < W - 1)   // the first W-1 dpre complete dx of the row group below
                ct_st<float, P>(xb + (rg * CT_HALO + i) * CC + col * P, dp);
#pragma unroll
            for (int kk = 0; kk < W - 1; ++kk)
#pragma unroll
                for (int q = 0; q < P; ++q) {
                    win[kk][q] = win[kk + 1][q];
                    dq[kk][q] = dq[kk + 1][q];
                }
#pragma unroll
            for (int q = 0; q < P; ++q) dq[W - 1][q] = dp[q];
            if (i >= W - 1) {
                cv_dx_emit<T, W, P>(wk, dq, valid && t0 + r0 + i - (W - 1) < L, dx + ((int64_t)b * L + t0 + r0 + i - (W - 1)) * D + c);
            } else if (emit_prev) {   // dx at t = i - (W-1) < 0 is dx_prev[i] (dpre before 0 is zero)
                cv_dx_emit<T, W, P>(wk, dq, true, dx_prev + ((int64_t)b * (W - 1) + i) * D + c);
            }
        }
        float nx[CT_HALO][P];   // dpre of the W-1 rows after this thread's rows
        if (rg == G - 1) {
#pragma unroll
            for (int i = 0; i < W - 1; ++i) {
                float g[P];
                ct_ld<T, P>(sx + (CT_TT + CT_HALO + i) * CC, win[W - 1]);
                ct_ld<T, P>(sg + (CT_TT + i) * CC, g);
                cv_dpre<P, W>(wk, bv, win, g, act, nx[i]);
#pragma unroll
                for (int kk = 0; kk < W - 1; ++kk)
#pragma unroll
                    for (int q = 0; q < P; ++q) win[kk][q] = win[kk + 1][q];
            }
        }
        __syncwarp();
        if (lane == 0) cv_arrive(&empty[st]);   // the stage is no longer read
        if (cv_bar_any(!ok)) break;
        if (rg < G - 1) {
#pragma unroll
            for (int i = 0; i < W - 1; ++i) {
                ct_ld<float, P>(xb + ((rg + 1) * CT_HALO + i) * CC + col * P, nx[i]);
            }
        }
        // the last W-1 rows of the thread
#pragma unroll
        for (int i = 0; i < W - 1; ++i) {
#pragma unroll
            for (int kk = 0; kk < W - 1; ++kk)
#pragma unroll
                for (int q = 0; q < P; ++q) dq[kk][q] = dq[kk + 1][q];
#pragma unroll
            for (int q = 0; q < P; ++q) dq[W - 1][q] = nx[i][q];
            const int t = t0 + r0 + R - (W - 1) + i;
            cv_dx_emit<T, W, P>(wk, dq, valid && t < L, dx + ((int64_t)b * L + t) * D + c);
        }
    }
    // dweight / dbias of this CTA: sum the row groups in order through shared memory (the ring
    // is free: every consumer has passed its last stage), then one partial per (seg, tap, channel)
    cv_bar();
    float* red = reinterpret_cast<float*>(cv_smem);   // [G][W + 1][CC]
#pragma unroll
    for (int kk = 0; kk < W; ++kk)
        ct_st<float, P>(red + (rg * (W + 1) + kk) * CC + col * P, aw[kk]);
    ct_st<float, P>(red + (rg * (W + 1) + W) * CC + col * P, ab);
    cv_bar();
    for (int idx = tid; idx < (W + 1) * CC; idx += CT_THREADS) {
        const int kk = idx / CC, ch = idx % CC, d = cb * CC + ch;
        float s = 0.f;
        for (int g = 0; g < G; ++g) s += red[(g * (W + 1) + kk) * CC + ch];
        if (d < D) part[((int64_t)seg * (W + 1) + kk) * D + d] = s;
    }
}

static int cv_fail(int code, const char* fmt, ...) {
    char buf[256];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    return report_error(code, buf);
}

template <typename T, int VEC, int W>
static cudaError_t cv_fwd_launch(const void* x, const void* w, const void* bias, const void* x_prev, int act, void* y,
                                 int64_t B, int64_t L, int64_t D, cudaStream_t s) {
    const int64_t groups = (D + VEC - 1) / VEC;
    dim3 grid((unsigned)((groups + CV_THREADS - 1) / CV_THREADS), (unsigned)((L + CV_RUN - 1) / CV_RUN), (unsigned)B);
    conv1d_fwd_kernel<T, VEC, W><<<grid, CV_THREADS, 0, s>>>(
        static_cast<const T*>(x), static_cast<const T*>(w), static_cast<const T*>(bias),
        static_cast<const T*>(x_prev), act, static_cast<T*>(y), L, D);
    return cudaGetLastError();
}

template <typename T, int VEC, int W>
static cudaError_t cv_bwd_launch(const void* x, const void* w, const void* bias, const void* x_prev, int act,
                                 const void* dy, void* dx, void* dw, void* db, void* dx_prev, float* part,
                                 int64_t B, int64_t L, int64_t D, cudaStream_t s) {
    const int64_t groups = (D + VEC - 1) / VEC;
    const int64_t nrun = (L + CV_RUN - 1) / CV_RUN;
    dim3 grid((unsigned)((groups + CV_THREADS - 1) / CV_THREADS), (unsigned)nrun, (unsigned)B);
    conv1d_bwd_kernel<T, VEC, W><<<grid, CV_THREADS, 0, s>>>(
        static_cast<const T*>(x), static_cast<const T*>(w), static_cast<const T*>(bias),
        static_cast<const T*>(x_prev), act, static_cast<const T*>(dy), static_cast<T*>(dx),
        static_cast<T*>(dx_prev), part, L, D, nrun);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const int64_t n = (int64_t)(W + 1) * D;
    conv1d_reduce_kernel<T, W><<<(unsigned)((n + 255) / 256), 256, 0, s>>>(part, B * nrun, D, static_cast<T*>(dw),
                                                                          static_cast<T*>(db));
    return cudaGetLastError();
}

template <typename T, int W>
static cudaError_t cv_fwd_w(bool vec, const void* x, const void* w, const void* bias, const void* x_prev, int act,
                            void* y, int64_t B, int64_t L, int64_t D, cudaStream_t s) {
    constexpr int V = 16 / (int)sizeof(T);
    return vec ? cv_fwd_launch<T, V, W>(x, w, bias, x_prev, act, y, B, L, D, s)
               : cv_fwd_launch<T, 1, W>(x, w, bias, x_prev, act, y, B, L, D, s);
}

template <typename T, int W>
static cudaError_t cv_bwd_w(bool vec, const void* x, const void* w, const void* bias, const void* x_prev, int act,
                            const void* dy, void* dx, void* dw, void* db, void* dx_prev, float* part, int64_t B,
                            int64_t L, int64_t D, cudaStream_t s) {
    constexpr int V = 16 / (int)sizeof(T);
    return vec ? cv_bwd_launch<T, V, W>(x, w, bias, x_prev, act, dy, dx, dw, db, dx_prev, part, B, L, D, s)
               : cv_bwd_launch<T, 1, W>(x, w, bias, x_prev, act, dy, dx, dw, db, dx_prev, part, B, L, D, s);
}

template <typename T>
static cudaError_t cv_fwd_t(int W, bool vec, const void* x, const void* w, const void* bias, const void* x_prev,
                            int act, void* y, int64_t B, int64_t L, int64_t D, cudaStream_t s) {
    switch (W) {
        case 1: return cv_fwd_w<T, 1>(vec, x, w, bias, x_prev, act, y, B, L, D, s);
        case 2: return cv_fwd_w<T, 2>(vec, x, w, bias, x_prev, act, y, B, L, D, s);
        case 3: return cv_fwd_w<T, 3>(vec, x, w, bias, x_prev, act, y, B, L, D, s);
        default: return cv_fwd_w<T, 4>(vec, x, w, bias, x_prev, act, y, B, L, D, s);
    }
}

template <typename T>
static cudaError_t cv_bwd_t(int W, bool vec, const void* x, const void* w, const void* bias, const void* x_prev,
                            int act, const void* dy, void* dx, void* dw, void* db, void* dx_prev, float* part,
                            int64_t B, int64_t L, int64_t D, cudaStream_t s) {
    switch (W) {
        case 1: return cv_bwd_w<T, 1>(vec, x, w, bias, x_prev, act, dy, dx, dw, db, dx_prev, part, B, L, D, s);
        case 2: return cv_bwd_w<T, 2>(vec, x, w, bias, x_prev, act, dy, dx, dw, db, dx_prev, part, B, L, D, s);
        case 3: return cv_bwd_w<T, 3>(vec, x, w, bias, x_prev, act, dy, dx, dw, db, dx_prev, part, B, L, D, s);
        default: return cv_bwd_w<T, 4>(vec, x, w, bias, x_prev, act, dy, dx, dw, db, dx_prev, part, B, L, D, s);
    }
}

static bool cv_aligned16(const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---- TMA-staged path (rows 16-byte aligned, sizes within int32, tensor maps encodable)

template <typename T, int W>
static cudaError_t ct_fwd_launch(const CUtensorMap& tm, const void* w, const void* bias, const void* x_prev, int act,
                                 void* y, int B, int L, int D, int sms, cudaStream_t s) {
    constexpr int CC = CtShape<T, CT_FWD_CPT>::CC;
    const int ncb = (D + CC - 1) / CC;
    const int nitems = B * ((L + CT_TT - 1) / CT_TT);
    const int nseg = std::max(1, std::min(nitems, sms * CT_FWD_CTAS_PER_SM / ncb));
    const size_t smem = (size_t)CT_FWD_ST * (CT_TT + CT_HALO) * CT_ROWB + 2 * CT_FWD_ST * sizeof(uint64_t);
    auto kern = conv1d_fwd_tma_kernel<T, W>;
    cudaError_t e = ensure_smem_attr<conv1d_fwd_tma_kernel<T, W>>((int)smem);
    if (e != cudaSuccess) return e;
    kern<<<(unsigned)ncb * nseg, CT_THREADS + 32, smem, s>>>(
        tm, static_cast<const T*>(w), static_cast<const T*>(bias), static_cast<const T*>(x_prev), act,
        static_cast<T*>(y), B, L, D, ncb, nseg);
    return cudaGetLastError();
}

// Number of backward CTAs per channel block (= dweight / dbias partials per channel).
static int ct_bwd_segments(int64_t B, int64_t L, int64_t D, int cc) {
    const int64_t ncb = (D + cc - 1) / cc;
    const int64_t nitems = B * ((L + CT_TT - 1) / CT_TT);
    return (int)std::max<int64_t>(1, std::min<int64_t>(nitems, CT_BWD_CTAS / ncb));
}

template <typename T, int W>
static cudaError_t ct_bwd_launch(const CUtensorMap& tmx, const CUtensorMap& tmg, const void* w, const void* bias,
                                 const void* x_prev, int act, void* dx, void* dw, void* db, void* dx_prev, float* part,
                                 int B, int L, int D, cudaStream_t s) {
    using Sh = CtShape<T, CT_BWD_CPT>;
    const int ncb = (D + Sh::CC - 1) / Sh::CC;
    const int nseg = ct_bwd_segments(B, L, D, Sh::CC);
    const size_t smem = (size_t)CT_BWD_ST * ((CT_TT + 2 * CT_HALO) + (CT_TT + CT_HALO)) * CT_ROWB +
                        2 * (size_t)Sh::G * CT_HALO * Sh::CC * sizeof(float) + 2 * CT_BWD_ST * sizeof(uint64_t);
    auto kern = conv1d_bwd_tma_kernel<T, W>;
    cudaError_t e = ensure_smem_attr<conv1d_bwd_tma_kernel<T, W>>((int)smem);
    if (e != cudaSuccess) return e;
    kern<<<(unsigned)ncb * nseg, CT_THREADS + 32, smem, s>>>(
        tmx, tmg, static_cast<const T*>(w), static_cast<const T*>(bias), static_cast<const T*>(x_prev), act,
        static_cast<T*>(dx), static_cast<T*>(dx_prev), part, B, L, D, ncb, nseg);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const int64_t n = (int64_t)(W + 1) * D;
    conv1d_reduce_kernel<T, W><<<(unsigned)((n + 255) / 256), 256, 0, s>>>(part, nseg, D, static_cast<T*>(dw),
                                                                          static_cast<T*>(db));
    return cudaGetLastError();
}

template <typename T>
static cudaError_t ct_fwd_t(int W, const CUtensorMap& tm, const void* w, const void* bias, const void* x_prev, int act,
                            void* y, int B, int L, int D, int sms, cudaStream_t s) {
    switch (W) {
        case 1: return ct_fwd_launch<T, 1>(tm, w, bias, x_prev, act, y, B, L, D, sms, s);
        case 2: return ct_fwd_launch<T, 2>(tm, w, bias, x_prev, act, y, B, L, D, sms, s);
        case 3: return ct_fwd_launch<T, 3>(tm, w, bias, x_prev, act, y, B, L, D, sms, s);
        default: return ct_fwd_launch<T, 4>(tm, w, bias, x_prev, act, y, B, L, D, sms, s);
    }
}

template <typename T>
static cudaError_t ct_bwd_t(int W, const CUtensorMap& tmx, const CUtensorMap& tmg, const void* w, const void* bias,
                            const void* x_prev, int act, void* dx, void* dw, void* db, void* dx_prev, float* part,
                            int B, int L, int D, cudaStream_t s) {
    switch (W) {
        case 1: return ct_bwd_launch<T, 1>(tmx, tmg, w, bias, x_prev, act, dx, dw, db, dx_prev, part, B, L, D, s);
        case 2: return ct_bwd_launch<T, 2>(tmx, tmg, w, bias, x_prev, act, dx, dw, db, dx_prev, part, B, L, D, s);
        case 3: return ct_bwd_launch<T, 3>(tmx, tmg, w, bias, x_prev, act, dx, dw, db, dx_prev, part, B, L, D, s);
        default: return ct_bwd_launch<T, 4>(tmx, tmg, w, bias, x_prev, act, dx, dw, db, dx_prev, part, B, L, D, s);
    }
}

static bool ct_sizes_ok(int64_t B, int64_t L, int64_t D, int64_t es) {
    return (D * es) % 16 == 0 && B <= 0x7fffffffLL && L <= 0x7fffffffLL - 2 * CT_TT && D <= 0x7fffffffLL &&
           B * ((L + CT_TT - 1) / CT_TT) <= 0x7fffffffLL;
}

static const int* ct_err_word() {
    static std::atomic<const int*> cache[64];   // per device ordinal
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    if (dev >= 0 && dev < 64) {
        const int* w = cache[dev].load(std::memory_order_relaxed);
        if (w != nullptr) return w;
    }
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_cv_err) != cudaSuccess) return nullptr;
    if (dev >= 0 && dev < 64) cache[dev].store(static_cast<const int*>(p), std::memory_order_relaxed);
    return static_cast<const int*>(p);
}

static int cv_check(int dtype, int64_t B, int64_t L, int64_t D, int64_t W, int act) {
    if (dtype != MWC_F32 && dtype != MWC_F16 && dtype != MWC_BF16)
        return cv_fail(MWC_ERR_INVALID, "x must be float32/float16/bfloat16 (dtype code %d)", dtype);
    if (B < 0 || L < 0 || D < 0) return cv_fail(MWC_ERR_INVALID, "negative size");
    if (W < 1 || W > 4) return cv_fail(MWC_ERR_UNSUPPORTED, "kernel width must be 1..4 (got %lld)", (long long)W);
    if (act != 0 && act != 1) return cv_fail(MWC_ERR_INVALID, "activation must be 0 (none) or 1 (silu)");
    if (B > 65535 || (L + CV_RUN - 1) / CV_RUN > 65535) return cv_fail(MWC_ERR_UNSUPPORTED, "shape too large");
    return MWC_OK;
}

}  // namespace mwc

using namespace mwc;

extern "C" {

int mwc_conv1d_fwd(const void* x, const void* weight, const void* bias, const void* x_prev, int activation,
                   void* y, int64_t B, int64_t L, int64_t D, int64_t W, int dtype, void* stream) {
    int rc = cv_check(dtype, B, L, D, W, activation);
    if (rc != MWC_OK) return rc;
    if (!x || !weight || !y) return cv_fail(MWC_ERR_INVALID, "x, weight and y are required");
    if (B == 0 || L == 0 || D == 0) return report_ok();
    const int64_t es = dtype == MWC_F32 ? 4 : 2;
    const bool vec = (D * es) % 16 == 0 && cv_aligned16(x) && cv_aligned16(y) && cv_aligned16(x_prev);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    note_err_word(nullptr);
    CUtensorMap tm;
    if (vec && ct_sizes_ok(B, L, D, es) && make_tmap_3d(&tm, x, dtype, D, L, B, CT_ROWB / (int)es, CT_TT + CT_HALO)) {
        const int sms = current_device_sms();
        cudaError_t e = dtype == MWC_BF16
                            ? ct_fwd_t<__nv_bfloat16>((int)W, tm, weight, bias, x_prev, activation, y, (int)B, (int)L, (int)D, sms, s)
                        : dtype == MWC_F16
                            ? ct_fwd_t<__half>((int)W, tm, weight, bias, x_prev, activation, y, (int)B, (int)L, (int)D, sms, s)
                            : ct_fwd_t<float>((int)W, tm, weight, bias, x_prev, activation, y, (int)B, (int)L, (int)D, sms, s);
        if (e != cudaSuccess) return cv_fail(MWC_ERR_CUDA, "conv1d forward launch: %s", cudaGetErrorString(e));
        note_err_word(ct_err_word());
        return report_ok();
    }
    cudaError_t e = dtype == MWC_BF16 ? cv_fwd_t<__nv_bfloat16>((int)W, vec, x, weight, bias, x_prev, activation, y, B, L, D, s)
                    : dtype == MWC_F16 ? cv_fwd_t<__half>((int)W, vec, x, weight, bias, x_prev, activation, y, B, L, D, s)
                                       : cv_fwd_t<float>((int)W, vec, x, weight, bias, x_prev, activation, y, B, L, D, s);
    if (e != cudaSuccess) return cv_fail(MWC_ERR_CUDA, "conv1d forward launch: %s", cudaGetErrorString(e));
    return report_ok();
}

int64_t mwc_conv1d_bwd_workspace_bytes(int64_t B, int64_t L, int64_t D, int64_t W) {
    if (B <= 0 || L <= 0 || D <= 0 || W <= 0) return 0;
    // the larger of the two paths' partial sums: per (b, 64-step run), or per backward CTA of
    // the TMA path (at most the count for 16-bit channel blocks)
    const int64_t nrun = (L + CV_RUN - 1) / CV_RUN;
    const int64_t nparts = std::max<int64_t>(B * nrun, ct_bwd_segments(B, L, D, CtShape<__half, CT_BWD_CPT>::CC));
    return (nparts * (W + 1) * D * 4 + 255) / 256 * 256;
}

int mwc_conv1d_bwd(const void* x, const void* weight, const void* bias, const void* x_prev, int activation,
                   const void* dy, void* dx, void* dweight, void* dbias, void* dx_prev, void* workspace,
                   int64_t workspace_bytes, int64_t B, int64_t L, int64_t D, int64_t W, int dtype, void* stream) {
    int rc = cv_check(dtype, B, L, D, W, activation);
    if (rc != MWC_OK) return rc;
    if (!x || !weight || !dy || !dx || !dweight) return cv_fail(MWC_ERR_INVALID, "x, weight, dy, dx and dweight are required");
    const int64_t es = dtype == MWC_F32 ? 4 : 2;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (B == 0 || L == 0 || D == 0) {
        cudaError_t e = cudaSuccess;
        if (D > 0) e = cudaMemsetAsync(dweight, 0, (size_t)(D * W * es), s);
        if (e == cudaSuccess && dbias != nullptr && D > 0) e = cudaMemsetAsync(dbias, 0, (size_t)(D * es), s);
        if (e == cudaSuccess && dx_prev != nullptr && B > 0 && D > 0 && W > 1)
            e = cudaMemsetAsync(dx_prev, 0, (size_t)(B * (W - 1) * D * es), s);
        if (e != cudaSuccess) return cv_fail(MWC_ERR_CUDA, "conv1d backward: %s", cudaGetErrorString(e));
        return report_ok();
    }
    const int64_t need = mwc_conv1d_bwd_workspace_bytes(B, L, D, W);
    if (workspace == nullptr || workspace_bytes < need || !cv_aligned16(workspace))
        return cv_fail(MWC_ERR_WORKSPACE, "conv1d backward workspace of %lld bytes (16-byte aligned) required",
                       (long long)need);
    if (dx_prev != nullptr && W > 1 && L < W - 1)
        return cv_fail(MWC_ERR_UNSUPPORTED, "dx_prev needs L >= W - 1");
    const bool vec = (D * es) % 16 == 0 && cv_aligned16(x) && cv_aligned16(dy) && cv_aligned16(dx) &&
                     cv_aligned16(x_prev) && cv_aligned16(dx_prev);
    float* part = static_cast<float*>(workspace);
    void* dxp = W > 1 ? dx_prev : nullptr;
    note_err_word(nullptr);
    CUtensorMap tmx, tmg;
    if (vec && cv_aligned16(dweight) && ct_sizes_ok(B, L, D, es) &&
        make_tmap_3d(&tmx, x, dtype, D, L, B, CT_ROWB / (int)es, CT_TT + 2 * CT_HALO) &&
        make_tmap_3d(&tmg, dy, dtype, D, L, B, CT_ROWB / (int)es, CT_TT + CT_HALO)) {
        cudaError_t e = dtype == MWC_BF16
                            ? ct_bwd_t<__nv_bfloat16>((int)W, tmx, tmg, weight, bias, x_prev, activation, dx, dweight, dbias, dxp, part, (int)B, (int)L, (int)D, s)
                        : dtype == MWC_F16
                            ? ct_bwd_t<__half>((int)W, tmx, tmg, weight, bias, x_prev, activation, dx, dweight, dbias, dxp, part, (int)B, (int)L, (int)D, s)
                            : ct_bwd_t<float>((int)W, tmx, tmg, weight, bias, x_prev, activation, dx, dweight, dbias, dxp, part, (int)B, (int)L, (int)D, s);
        if (e != cudaSuccess) return cv_fail(MWC_ERR_CUDA, "conv1d backward launch: %s", cudaGetErrorString(e));
        note_err_word(ct_err_word());
        return report_ok();
    }
    cudaError_t e = dtype == MWC_BF16
                        ? cv_bwd_t<__nv_bfloat16>((int)W, vec, x, weight, bias, x_prev, activation, dy, dx, dweight, dbias, dxp, part, B, L, D, s)
                    : dtype == MWC_F16
                        ? cv_bwd_t<__half>((int)W, vec, x, weight, bias, x_prev, activation, dy, dx, dweight, dbias, dxp, part, B, L, D, s)
                        : cv_bwd_t<float>((int)W, vec, x, weight, bias, x_prev, activation, dy, dx, dweight, dbias, dxp, part, B, L, D, s);
    if (e != cudaSuccess) return cv_fail(MWC_ERR_CUDA, "conv1d backward launch: %s", cudaGetErrorString(e));
    return report_ok();
}

}  // extern "C"
