// First-order linear recurrence h_t = a_t h_{t-1} + x_t along L for (R, L, N) tensors
// (parallel_scan_fn, mamba_windows_cuda/pscan.py:139-150, with the semantics of
// parallel_scan_ref, pscan.py:153-171: h_0 = x_0, a_0 ignored), and its gradient.
//
// One warp scans one row for G adjacent columns: lane = (slice, column), each lane holds
// K consecutive time steps in registers. A pass covers 32/G * K steps: each lane reduces
// its K steps to an affine map (P, S) (h_out = P h_in + S), a warp-shuffle scan composes
// the maps across slices, and the running carry links consecutive passes. HBM-bound:
// a and x are read once, h written once.
#include "mwc_device.cuh"
#include "mwc_internal.h"

namespace mwc {

constexpr int LIN_WARPS = 4;

template <typename T, int K>
struct VecIO {
    static_assert(K * sizeof(T) == 16, "one 16-byte vector per lane");
    __device__ __forceinline__ static void load(float (&v)[K], const T* src) {
        uint4 raw = __ldg(reinterpret_cast<const uint4*>(src));
        const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
        for (int k = 0; k < K; ++k) v[k] = to_f(e[k]);
    }
    __device__ __forceinline__ static void store(T* dst, const float (&v)[K]) {
        uint4 raw;
        T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
        for (int k = 0; k < K; ++k) e[k] = from_f<T>(v[k]);
        *reinterpret_cast<uint4*>(dst) = raw;
    }
};

template <typename T, int G, int K>
__global__ void __launch_bounds__(LIN_WARPS * 32) lin_fwd_kernel(const LinArgs p) {
    constexpr int NS = 32 / G;
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int nl = lane % G, sl = lane / G;
    const int64_t r = (int64_t)blockIdx.x * LIN_WARPS + warp;
    if (r >= p.R) return;  // whole warp
    const int64_t n = (int64_t)blockIdx.y * G + nl;
    const bool nv = n < p.N;
    const int64_t base = r * p.L * p.N;
    const T* a = static_cast<const T*>(p.a) + base;
    const T* x = static_cast<const T*>(p.x) + base;
    T* h = static_cast<T*>(p.out_h) + base;
    const bool vec = (G == 1) && (p.vec != 0) && (K * sizeof(T) == 16);
    float carry = 0.f;
    for (int64_t t0 = 0; t0 < p.L; t0 += NS * K) {
        const int64_t tl = t0 + (int64_t)sl * K;
        float av[K], xv[K];
        const bool full = vec && (tl + K <= p.L);
        if constexpr (G == 1 && K * sizeof(T) == 16) {
            if (full) {
                VecIO<T, K>::load(av, a + tl);
                VecIO<T, K>::load(xv, x + tl);
            }
        }
        if (!full) {
#pragma unroll
            for (int k = 0; k < K; ++k) {
                const int64_t t = tl + k;
                const bool ok = nv && t < p.L;
                av[k] = ok ? to_f(a[t * p.N + n]) : 1.f;
                xv[k] = ok ? to_f(x[t * p.N + n]) : 0.f;
            }
        }
        if (tl == 0) av[0] = 0.f;  // h_0 = x_0
        float P = 1.f, S = 0.f, loc[K], pc[K];
#pragma unroll
        for (int k = 0; k < K; ++k) {
            S = fmaf(av[k], S, xv[k]);
            P *= av[k];
            loc[k] = S;
            pc[k] = P;
        }
#pragma unroll
        for (int off = 1; off < NS; off <<= 1) {
            const float Pp = __shfl_up_sync(FULL, P, off * G);
            const float Sp = __shfl_up_sync(FULL, S, off * G);
            if (sl >= off) {
                S = fmaf(P, Sp, S);
                P *= Pp;
            }
        }
        float Pe = __shfl_up_sync(FULL, P, G);
        float Se = __shfl_up_sync(FULL, S, G);
        if (sl == 0) {
            Pe = 1.f;
            Se = 0.f;
        }
        const float hin = fmaf(Pe, carry, Se);
        float hv[K];
#pragma unroll
        for (int k = 0; k < K; ++k) hv[k] = fmaf(pc[k], hin, loc[k]);
        if constexpr (G == 1 && K * sizeof(T) == 16) {
            if (full) VecIO<T, K>::store(h + tl, hv);
        }
        if (!full) {
#pragma unroll
            for (int k = 0; k < K; ++k) {
                const int64_t t = tl + k;
                if (nv && t < p.L) h[t * p.N + n] = from_f<T>(hv[k]);
            }
        }
        const float Pt = __shfl_sync(FULL, P, (NS - 1) * G + nl);
        const float St = __shfl_sync(FULL, S, (NS - 1) * G + nl);
        carry = fmaf(Pt, carry, St);
    }
}

// z_t = a_{t+1} z_{t+1} + g_t (a_L = 0) run backwards; gx = z, ga_t = z_t h_{t-1}, ga_0 = 0.
template <typename T, int G, int K>
__global__ void __launch_bounds__(LIN_WARPS * 32) lin_bwd_kernel(const LinArgs p) {
    constexpr int NS = 32 / G;
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int nl = lane % G, sl = lane / G;
    const int64_t r = (int64_t)blockIdx.x * LIN_WARPS + warp;
    if (r >= p.R) return;
    const int64_t n = (int64_t)blockIdx.y * G + nl;
    const bool nv = n < p.N;
    const int64_t base = r * p.L * p.N;
    const T* a = static_cast<const T*>(p.a) + base;
    const T* hh = static_cast<const T*>(p.h) + base;
    const T* g = static_cast<const T*>(p.g) + base;
    T* ga = static_cast<T*>(p.ga) + base;
    T* gx = static_cast<T*>(p.gx) + base;
    const int64_t span = (int64_t)NS * K;
    const int64_t npass = (p.L + span - 1) / span;
    float carry = 0.f;
    for (int64_t pi = npass - 1; pi >= 0; --pi) {
        const int64_t tl = pi * span + (int64_t)sl * K;
        float cv[K], gv[K], hv[K];
#pragma unroll
        for (int k = 0; k < K; ++k) {
            const int64_t t = tl + k;
            const bool ok = nv && t < p.L;
            cv[k] = (ok && t + 1 < p.L) ? to_f(a[(t + 1) * p.N + n]) : 0.f;
            gv[k] = ok ? to_f(g[t * p.N + n]) : 0.f;
            hv[k] = (ok && t >= 1) ? to_f(hh[(t - 1) * p.N + n]) : 0.f;
        }
        float P = 1.f, S = 0.f, loc[K], pc[K];
#pragma unroll
        for (int k = K - 1; k >= 0; --k) {
            S = fmaf(cv[k], S, gv[k]);
            P *= cv[k];
            loc[k] = S;
            pc[k] = P;
        }
#pragma unroll
        for (int off = 1; off < NS; off <<= 1) {
            const float Pn = __shfl_down_sync(FULL, P, off * G);
            const float Sn = __shfl_down_sync(FULL, S, off * G);
            if (sl + off < NS) {
                S = fmaf(P, Sn, S);
                P *= Pn;
            }
        }
        float Pe = __shfl_down_sync(FULL, P, G);
        float Se = __shfl_down_sync(FULL, S, G);
        if (sl == NS - 1) {
            Pe = 1.f;
            Se = 0.f;
        }
        const float zin = fmaf(Pe, carry, Se);
#pragma unroll
        for (int k = 0; k < K; ++k) {
            const int64_t t = tl + k;
            if (nv && t < p.L) {
                const float z = fmaf(pc[k], zin, loc[k]);
                gx[t * p.N + n] = from_f<T>(z);
                ga[t * p.N + n] = from_f<T>(z * hv[k]);
            }
        }
        const float Pt = __shfl_sync(FULL, P, nl);
        const float St = __shfl_sync(FULL, S, nl);
        carry = fmaf(Pt, carry, St);
    }
}

static int pick_group(int64_t N) {
    int G = 1;
    while (G < N && G < 32) G <<= 1;
    return G;
}

template <typename T, int G>
static void launch_lin_g(const LinArgs& a, bool fwd, cudaStream_t s) {
    constexpr int K = (G == 1) ? (int)(16 / sizeof(T)) : 4;
    dim3 grid((unsigned)((a.R + LIN_WARPS - 1) / LIN_WARPS), (unsigned)((a.N + G - 1) / G), 1);
    if (fwd) lin_fwd_kernel<T, G, K><<<grid, LIN_WARPS * 32, 0, s>>>(a);
    else lin_bwd_kernel<T, G, K><<<grid, LIN_WARPS * 32, 0, s>>>(a);
}

template <typename T>
static cudaError_t launch_lin_t(const LinArgs& a, bool fwd, cudaStream_t s) {
    switch (pick_group(a.N)) {
        case 1: launch_lin_g<T, 1>(a, fwd, s); break;
        case 2: launch_lin_g<T, 2>(a, fwd, s); break;
        case 4: launch_lin_g<T, 4>(a, fwd, s); break;
        case 8: launch_lin_g<T, 8>(a, fwd, s); break;
        case 16: launch_lin_g<T, 16>(a, fwd, s); break;
        default: launch_lin_g<T, 32>(a, fwd, s); break;
    }
    return cudaGetLastError();
}

cudaError_t launch_lin_fwd(const LinArgs& a, int dtype, cudaStream_t s) {
    if (dtype == 2) return launch_lin_t<__nv_bfloat16>(a, true, s);
    return dtype == 1 ? launch_lin_t<__half>(a, true, s) : launch_lin_t<float>(a, true, s);
}

cudaError_t launch_lin_bwd(const LinArgs& a, int dtype, cudaStream_t s) {
    if (dtype == 2) return launch_lin_t<__nv_bfloat16>(a, false, s);
    return dtype == 1 ? launch_lin_t<__half>(a, false, s) : launch_lin_t<float>(a, false, s);
}

}  // namespace mwc
