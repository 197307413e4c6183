// Forward selective scan for sm_100a: fused discretisation (ex2 with log2(e) folded into
// A), recurrence, C.h + D.u epilogue, h_prev in / h_last out, float32 checkpoints every
// 16 steps for the backward, and the L-segmented mode (segment scans from zero + carry
// fold + truncated fixup) used when batch x channels cannot fill the GPU.
//
// Thread layout: a channel's N states (N = 16, the reference's; 32 / 64 for the forward of
// mwc_ss_fwd_nstate) are split over P = N/S lanes (S states each, held in registers). Lanes
// of one warp cover 32/P channels, consecutive lanes consecutive channels, so the (B, L, D)
// tiles are read and written along D. Tiles of u / delta (LT x channels) and the B / C rows
// (LT x N, float32) are staged in shared memory.
//
// Reference semantics: selective_scan_fwd_kernel_v4 (mamba_windows_cuda/mamba_cuda.py:93-174)
// and selective_scan_fwd_store_kernel (:611-667): a = safe_exp(delta*A) with the exponent
// clamped at 88 (:65-70), h = a h + (delta u) B, y = sum_n C_n h_n + u D.
#include "mwc_device.cuh"
#include "mwc_internal.h"

#include <algorithm>

namespace mwc {

constexpr int FWD_LT = 16;  // time steps per shared-memory tile (a multiple of CK)
constexpr int FWD_NW = 4;   // warps per CTA

// a[j] = 2^(dt*A2[j]), exponent clamped above at 88*log2(e) like safe_exp. The clamp is a
// per-thread branch taken only when some exponent can exceed it (A*delta > 88).
template <int S>
__device__ __forceinline__ void decay_factors(float (&a)[S], const float (&A2)[S], float dt,
                                              float a2max) {
    if (dt * a2max > ARG2_HI) {
#pragma unroll
        for (int j = 0; j < S; ++j) a[j] = ex2(fminf(dt * A2[j], ARG2_HI));
    } else {
#pragma unroll
        for (int j = 0; j < S; ++j) a[j] = ex2(dt * A2[j]);
    }
}

template <typename T, int N, int S, int NW>
__global__ void __launch_bounds__(NW * 32) ss_fwd_kernel(const FwdArgs p) {
    constexpr int P = N / S;   // lanes per channel
    constexpr int CPW = 32 / P;     // channels per warp
    constexpr int CPB = NW * CPW;   // channels per CTA
    constexpr int NT = NW * 32;
    constexpr int LT = FWD_LT;
    __shared__ __align__(16) T su[LT][CPB];
    __shared__ __align__(16) T sd[LT][CPB];
    __shared__ __align__(16) T sy[LT][CPB];
    __shared__ __align__(16) float sB[LT][N];
    __shared__ __align__(16) float sC[LT][N];

    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int sg = lane % P;
    const int cib = warp * CPW + lane / P;
    const int64_t d0 = (int64_t)blockIdx.x * CPB;
    const int64_t d = d0 + cib;
    const bool dv = d < p.D;
    const int64_t b = blockIdx.y;
    const int seg = blockIdx.z;
    const int64_t tbeg = (int64_t)seg * p.seg_len;
    const int64_t tend = min(tbeg + p.seg_len, p.L);
    const int ncols = (int)min((int64_t)CPB, p.D - d0);
    const bool vec = p.vec != 0;

    const T* Ap = static_cast<const T*>(p.A);
    float A2[S], h[S];
    float a2max = -INFINITY;
#pragma unroll
    for (int j = 0; j < S; ++j) {
        A2[j] = dv ? to_f(Ap[d * N + sg * S + j]) * LOG2E : 0.f;
        a2max = fmaxf(a2max, A2[j]);
        h[j] = 0.f;
    }
    const float Dd = dv ? to_f(static_cast<const T*>(p.Dv)[d]) : 0.f;
    if (seg == 0 && p.h_prev != nullptr && dv) {
        const T* hp = static_cast<const T*>(p.h_prev) + (b * p.D + d) * N + sg * S;
#pragma unroll
        for (int j = 0; j < S; ++j) h[j] = to_f(hp[j]);
    }

    const T* ub = static_cast<const T*>(p.u) + b * p.L * p.D + d0;
    const T* db = static_cast<const T*>(p.delta) + b * p.L * p.D + d0;
    const T* Bb = static_cast<const T*>(p.Bm) + b * p.L * N;
    const T* Cb = static_cast<const T*>(p.Cm) + b * p.L * N;
    T* yb = p.out ? static_cast<T*>(p.out) + b * p.L * p.D + d0 : nullptr;
    float sumd = 0.f;

    for (int64_t t0 = tbeg; t0 < tend; t0 += LT) {
        const int nrows = (int)min((int64_t)LT, tend - t0);
        __syncthreads();
        load_tile<T, LT, CPB, NT>(su, ub + t0 * p.D, p.D, nrows, ncols, vec);
        load_tile<T, LT, CPB, NT>(sd, db + t0 * p.D, p.D, nrows, ncols, vec);
        load_tile_f32<T, LT, N, NT>(sB, Bb + t0 * N, N, nrows);
        if (yb) load_tile_f32<T, LT, N, NT>(sC, Cb + t0 * N, N, nrows);
        __syncthreads();
        // Rows past the end are zero-filled: delta = 0 gives a = 1 and no input, so the
        // state is unchanged and no per-step bound check is needed.
#pragma unroll
        for (int i = 0; i < LT; ++i) {
            const float dt = to_f(sd[i][cib]);
            const float uu = to_f(su[i][cib]);
            const float du = dt * uu;
            sumd += dt;
            float a[S];
            decay_factors<S>(a, A2, dt, a2max);
            float yp = 0.f;
#pragma unroll
            for (int j = 0; j < S; ++j) {
                h[j] = fmaf(a[j], h[j], du * sB[i][sg * S + j]);
                yp = fmaf(sC[i][sg * S + j], h[j], yp);
            }
            if (yb) {
#pragma unroll
                for (int o = P / 2; o > 0; o >>= 1) yp += __shfl_xor_sync(FULL, yp, o);
                if (sg == 0) sy[i][cib] = from_f<T>(fmaf(Dd, uu, yp));
            }
            if ((i + 1) % CK == 0 && p.ckpt != nullptr) {
                const int64_t k = (t0 + i + 1) / CK - 1;
                if (k < p.nck && dv) {
                    float* c = p.ckpt + ((b * p.nck + k) * p.D + d) * N + sg * S;
#pragma unroll
                    for (int j = 0; j < S; ++j) c[j] = h[j];
                }
            }
        }
        if (yb) {
            __syncthreads();
            store_tile<T, LT, CPB, NT>(yb + t0 * p.D, sy, p.D, nrows, ncols, vec);
        }
    }

    if (!dv) return;
    if (p.nseg == 1) {
        if (p.h_last != nullptr) {
            T* hl = static_cast<T*>(p.h_last) + (b * p.D + d) * N + sg * S;
#pragma unroll
            for (int j = 0; j < S; ++j) hl[j] = from_f<T>(h[j]);
        }
        if (p.decay != nullptr) {
            float* dc = p.decay + (b * p.D + d) * N + sg * S;
#pragma unroll
            for (int j = 0; j < S; ++j) dc[j] = ex2(fminf(A2[j] * sumd, ARG2_HI));
        }
    } else {
        float* c = p.carry + ((b * p.nseg + seg) * p.D + d) * (N + 1);
#pragma unroll
        for (int j = 0; j < S; ++j) c[sg * S + j] = h[j];
        if (sg == 0) c[N] = sumd;
    }
}

// Carry fold + truncated fixup of a segment that was scanned from zero.
template <typename T, int N, int S, int NW>
__global__ void __launch_bounds__(NW * 32) ss_fixup_kernel(const FixupArgs p) {
    constexpr int P = N / S;
    constexpr int CPW = 32 / P;
    constexpr int CPB = NW * CPW;
    constexpr int NT = NW * 32;
    constexpr int LT = FWD_LT;
    __shared__ __align__(16) T sd[LT][CPB];
    __shared__ __align__(16) T sy[LT][CPB];
    __shared__ __align__(16) float sC[LT][N];

    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int sg = lane % P;
    const int cib = warp * CPW + lane / P;
    const int64_t d0 = (int64_t)blockIdx.x * CPB;
    const int64_t d = d0 + cib;
    const bool dv = d < p.D;
    const int64_t b = blockIdx.y;
    const int seg = (p.mode == 0) ? 1 + (int)blockIdx.z : (p.mode == 2 ? (int)blockIdx.z : 0);
    const int64_t tbeg = (int64_t)seg * p.seg_len;
    const int64_t tend = min(tbeg + p.seg_len, p.L);
    const int ncols = (int)min((int64_t)CPB, p.D - d0);
    const bool vec = p.vec != 0;
    const bool last = (p.mode == 1) || (p.mode == 2 && seg == 0) || (p.mode == 0 && seg == p.nseg - 1);

    const T* Ap = static_cast<const T*>(p.A);
    float A2[S], hin[S];
    float a2max = -INFINITY;
#pragma unroll
    for (int j = 0; j < S; ++j) {
        A2[j] = dv ? to_f(Ap[d * N + sg * S + j]) * LOG2E : 0.f;
        a2max = fmaxf(a2max, A2[j]);
        hin[j] = 0.f;
    }

    if (dv) {
        if (p.mode == 0) {
            // h_in(seg) = fold over earlier segments of (decay_s, S_s): h <- decay_s h + S_s
            for (int s = 0; s < seg; ++s) {
                const float* c = p.carry + ((b * p.nseg + s) * p.D + d) * (N + 1);
                const float sds = c[N];
#pragma unroll
                for (int j = 0; j < S; ++j)
                    hin[j] = fmaf(ex2(fminf(A2[j] * sds, ARG2_HI)), hin[j], c[sg * S + j]);
            }
            if (last) {
                const float* c = p.carry + ((b * p.nseg + seg) * p.D + d) * (N + 1);
                if (p.h_last != nullptr) {
                    T* hl = static_cast<T*>(p.h_last) + (b * p.D + d) * N + sg * S;
#pragma unroll
                    for (int j = 0; j < S; ++j)
                        hl[j] = from_f<T>(fmaf(ex2(fminf(A2[j] * c[N], ARG2_HI)), hin[j],
                                               c[sg * S + j]));
                }
                if (p.decay_out != nullptr) {
                    float tot = 0.f;
                    for (int s = 0; s < p.nseg; ++s)
                        tot += p.carry[((b * p.nseg + s) * p.D + d) * (N + 1) + N];
                    float* dc = p.decay_out + (b * p.D + d) * N + sg * S;
#pragma unroll
                    for (int j = 0; j < S; ++j) dc[j] = ex2(fminf(A2[j] * tot, ARG2_HI));
                }
            }
        } else {
            const float* hi = p.h_in + (b * p.D + d) * N + sg * S;
#pragma unroll
            for (int j = 0; j < S; ++j) hin[j] = hi[j];
            if (last && p.h_last != nullptr) {
                T* hl = static_cast<T*>(p.h_last) + (b * p.D + d) * N + sg * S;
                const float* dc = p.decay + (b * p.D + d) * N + sg * S;
#pragma unroll
                for (int j = 0; j < S; ++j) hl[j] = from_f<T>(fmaf(dc[j], hin[j], to_f(hl[j])));
            }
        }
    }
    if (p.out == nullptr && p.ckpt == nullptr) return;

    const T* db = static_cast<const T*>(p.delta) + b * p.L * p.D + d0;
    const T* Cb = static_cast<const T*>(p.Cm) + b * p.L * N;
    T* yb = p.out ? static_cast<T*>(p.out) + b * p.L * p.D + d0 : nullptr;
    float cum = 0.f;
    bool neg = false;
    if (p.mode == 2) {
        // chunk start: the delta prefix before the chunk; the chunk is skipped when every
        // state of every channel of the CTA stays below 2^-40 of h_in throughout it (the
        // minimum of the prefix over the chunk's steps bounds the largest factor exactly)
        const int64_t ntl = (p.L + DPRE_LT - 1) / DPRE_LT;
        const int64_t k0 = (int64_t)seg * FX_CHUNK_TILES;
        const int64_t k1 = min(k0 + FX_CHUNK_TILES, ntl);
        float cmin = INFINITY;
        if (dv) {
            const float* r = p.dpre + ((b * ntl + k0) * p.D + d) * 2;
            cum = r[0];
            for (int64_t k = k0; k < k1; ++k, r += p.D * 2) cmin = fminf(cmin, r[1]);
        }
        const bool skip = !dv || (a2max < 0.f && cmin * a2max < -40.f);
        if (__syncthreads_and(skip)) return;
    }
    for (int64_t t0 = tbeg; t0 < tend; t0 += LT) {
        const int nrows = (int)min((int64_t)LT, tend - t0);
        __syncthreads();
        load_tile<T, LT, CPB, NT>(sd, db + t0 * p.D, p.D, nrows, ncols, vec);
        if (yb) {
            load_tile<T, LT, CPB, NT>(sy, yb + t0 * p.D, p.D, nrows, ncols, vec);
            load_tile_f32<T, LT, N, NT>(sC, Cb + t0 * N, N, nrows);
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < LT; ++i) {
            const float dt = to_f(sd[i][cib]);
            cum += dt;
            neg |= dt < 0.f;
            float corr[S];
#pragma unroll
            for (int j = 0; j < S; ++j) corr[j] = ex2(fminf(A2[j] * cum, ARG2_HI)) * hin[j];
            if (yb) {
                float yp = 0.f;
#pragma unroll
                for (int j = 0; j < S; ++j) yp = fmaf(sC[i][sg * S + j], corr[j], yp);
#pragma unroll
                for (int o = P / 2; o > 0; o >>= 1) yp += __shfl_xor_sync(FULL, yp, o);
                if (sg == 0) sy[i][cib] = from_f<T>(to_f(sy[i][cib]) + yp);
            }
            if ((i + 1) % CK == 0 && p.ckpt != nullptr) {
                const int64_t k = (t0 + i + 1) / CK - 1;
                if (k < p.nck && dv) {
                    float* c = p.ckpt + ((b * p.nck + k) * p.D + d) * N + sg * S;
#pragma unroll
                    for (int j = 0; j < S; ++j) c[j] += corr[j];
                }
            }
        }
        if (yb) {
            __syncthreads();
            store_tile<T, LT, CPB, NT>(yb + t0 * p.D, sy, p.D, nrows, ncols, vec);
        }
        // Stop once every state of every channel in the CTA has decayed below 2^-40 of its
        // incoming value; with a non-negative delta stream it can only decay further.
        const bool done = !dv || (!neg && a2max < 0.f && cum * a2max < -40.f);
        if (__syncthreads_and(done)) break;
    }
}

// ---------------------------------------------------------------------------
// Host side: plan + launch
// ---------------------------------------------------------------------------

FwdPlan plan_fwd(int64_t B, int64_t L, int64_t D, int dtype, int num_sms) {
    (void)dtype;
    FwdPlan plan;
    const int64_t chans = B * D;
    // One lane per channel (S = 16) only when there are at least two such warps per SM
    // sub-partition; otherwise spread each channel over 4 lanes for finer-grained work.
    plan.states_per_thread = (chans >= (int64_t)num_sms * 4 * 32 * 2) ? 16 : 4;
    const int P = NSTATE / plan.states_per_thread;
    plan.channels_per_block = FWD_NW * (32 / P);
    const int64_t nblk = (D + plan.channels_per_block - 1) / plan.channels_per_block;
    const int64_t warps = nblk * B * FWD_NW;
    const int64_t target = (int64_t)num_sms * 16;  // four warps per SM sub-partition
    int nseg = 1;
    while (warps * nseg < target && (L / (2 * nseg)) >= 512) nseg *= 2;
    int64_t seg_len = (L + nseg - 1) / nseg;
    seg_len = ((seg_len + FWD_LT - 1) / FWD_LT) * FWD_LT;
    plan.seg_len = std::max<int64_t>(seg_len, FWD_LT);
    plan.nseg = (int)((L + plan.seg_len - 1) / plan.seg_len);
    if (plan.nseg < 1) plan.nseg = 1;
    return plan;
}

int64_t fwd_carry_floats(const FwdPlan& plan, int64_t B, int64_t D, int N) {
    return plan.nseg > 1 ? B * plan.nseg * D * (N + 1) : 0;
}

template <typename T, int N, int S>
static cudaError_t launch_fwd_t(const FwdArgs& a, const FwdPlan& plan, cudaStream_t s) {
    constexpr int CPB = FWD_NW * (32 / (N / S));
    dim3 grid((unsigned)((a.D + CPB - 1) / CPB), (unsigned)a.B, (unsigned)plan.nseg);
    ss_fwd_kernel<T, N, S, FWD_NW><<<grid, FWD_NW * 32, 0, s>>>(a);
    return cudaGetLastError();
}

template <typename T, int N, int S>
static cudaError_t launch_fixup_t(const FixupArgs& a, const FwdPlan& plan, cudaStream_t s) {
    constexpr int CPB = FWD_NW * (32 / (N / S));
    const unsigned gz = a.mode == 0 ? (unsigned)(plan.nseg - 1) : a.mode == 2 ? (unsigned)a.nseg : 1u;
    if (gz == 0) return cudaSuccess;
    dim3 grid((unsigned)((a.D + CPB - 1) / CPB), (unsigned)a.B, gz);
    ss_fixup_kernel<T, N, S, FWD_NW><<<grid, FWD_NW * 32, 0, s>>>(a);
    return cudaGetLastError();
}

// states per channel: 16 (the reference's N; also what N = 0 in the args means), 32 or 64
template <typename T, int N>
static cudaError_t launch_fwd_n(const FwdArgs& a, const FwdPlan& plan, cudaStream_t s) {
    switch (plan.states_per_thread) {
        case 16: return launch_fwd_t<T, N, 16>(a, plan, s);
        case 8: return launch_fwd_t<T, N, 8>(a, plan, s);
        default: return launch_fwd_t<T, N, 4>(a, plan, s);
    }
}

template <typename T>
static cudaError_t launch_fwd_s(const FwdArgs& a, const FwdPlan& plan, cudaStream_t s) {
    if (a.N == 64) return launch_fwd_n<T, 64>(a, plan, s);
    if (a.N == 32) return launch_fwd_n<T, 32>(a, plan, s);
    return launch_fwd_n<T, NSTATE>(a, plan, s);
}

template <typename T, int N>
static cudaError_t launch_fixup_n(const FixupArgs& a, const FwdPlan& plan, cudaStream_t s) {
    switch (plan.states_per_thread) {
        case 16: return launch_fixup_t<T, N, 16>(a, plan, s);
        case 8: return launch_fixup_t<T, N, 8>(a, plan, s);
        default: return launch_fixup_t<T, N, 4>(a, plan, s);
    }
}

template <typename T>
static cudaError_t launch_fixup_s(const FixupArgs& a, const FwdPlan& plan, cudaStream_t s) {
    if (a.N == 64) return launch_fixup_n<T, 64>(a, plan, s);
    if (a.N == 32) return launch_fixup_n<T, 32>(a, plan, s);
    return launch_fixup_n<T, NSTATE>(a, plan, s);
}

cudaError_t launch_fwd(const FwdArgs& a, const FwdPlan& plan, int dtype, cudaStream_t s) {
    if (dtype == 2) return launch_fwd_s<__nv_bfloat16>(a, plan, s);
    return dtype == 1 ? launch_fwd_s<__half>(a, plan, s) : launch_fwd_s<float>(a, plan, s);
}

cudaError_t launch_fixup(const FixupArgs& a, const FwdPlan& plan, int dtype, cudaStream_t s) {
    if (dtype == 2) return launch_fixup_s<__nv_bfloat16>(a, plan, s);
    return dtype == 1 ? launch_fixup_s<__half>(a, plan, s) : launch_fixup_s<float>(a, plan, s);
}

}  // namespace mwc
