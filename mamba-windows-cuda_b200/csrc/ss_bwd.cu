// Backward selective scan for sm_100a.
//
// Per CTA (one batch row, CPB channels) the sequence is walked backwards in chunks of
// CK = 16 steps. For each chunk the 16 forward states are recomputed from the float32
// checkpoint the forward wrote (or h_prev for the first chunk) and held in registers;
// the adjoint recurrence then runs backwards through the chunk:
//   g_t = dout_t C_t + q_{t+1},  q_t = a_t g_t              (q_L = dh_last)
//   du_t = dout_t D + dt_t <g_t, B_t>,  ddelta_t = <g_t, A a_t h_{t-1}> + u_t <g_t, B_t>
//   dA += g_t dt_t a_t h_{t-1},  dB_t = sum_d g_t dt_t u_t,  dC_t = sum_d dout_t h_t
//   dD += dout_t u_t,  dh_prev = q_0
// (the per-step terms of selective_scan_bwd_direct_kernel,
// mamba_windows_cuda/mamba_cuda.py:703-742, with h_{-1} = h_prev and dh_last added).
//
// Determinism: the reference adds dB/dC/dA/dD with float atomics. Here every sum has a
// fixed order: dB/dC over the channels of a warp by a butterfly reduce-scatter, over the
// warps of a CTA in warp order, over CTAs in the finalize kernel in block order; dA/dD
// per (batch, channel) in registers over time, then over batch in the finalize kernel.
#include "mwc_device.cuh"
#include "mwc_internal.h"

namespace mwc {

constexpr int BWD_NW = 4;   // warps per CTA
constexpr int BWD_S = 4;    // states per thread (4 lanes per channel)

// Reduce-scatter of V = 2S values across the CPW channel lanes of a warp (lanes that hold
// the same state group). Afterwards lane (chw, sg) holds the sum over the warp's channels
// of value index chw. Fixed pairing order -> bitwise reproducible.
template <int S, int P>
__device__ __forceinline__ float reduce_scatter_channels(float (&v)[2 * S], int chw) {
    constexpr int CPW = 32 / P;
    static_assert(2 * S == CPW, "one value per lane after the reduce-scatter");
#pragma unroll
    for (int m = CPW / 2; m >= 1; m >>= 1) {
        const bool up = (chw & m) != 0;
#pragma unroll
        for (int i = 0; i < m; ++i) {
            const float send = up ? v[i] : v[i + m];
            const float keep = up ? v[i + m] : v[i];
            v[i] = keep + __shfl_xor_sync(FULL, send, m * P);
        }
    }
    return v[0];
}

template <typename T, int S, int NW>
__global__ void __launch_bounds__(NW * 32) ss_bwd_kernel(const BwdArgs p) {
    constexpr int P = NSTATE / S;
    constexpr int CPW = 32 / P;
    constexpr int CPB = NW * CPW;
    constexpr int NT = NW * 32;
    constexpr int LT = CK;
    __shared__ __align__(16) T su[LT][CPB];
    __shared__ __align__(16) T sd[LT][CPB];
    __shared__ __align__(16) T sgy[LT][CPB];
    __shared__ __align__(16) T sdu[LT][CPB];
    __shared__ __align__(16) T sdd[LT][CPB];
    __shared__ __align__(16) float sB[LT][NSTATE];
    __shared__ __align__(16) float sC[LT][NSTATE];
    __shared__ __align__(16) float sred[NW][LT][2 * NSTATE];

    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int sg = lane % P;
    const int chw = lane / P;
    const int cib = warp * CPW + chw;
    const int64_t d0 = (int64_t)blockIdx.x * CPB;
    const int64_t d = d0 + cib;
    const bool dv = d < p.D;
    const int64_t b = blockIdx.y;
    const int ncols = (int)min((int64_t)CPB, p.D - d0);
    const bool vec = p.vec != 0;
    const int64_t Lp = (int64_t)p.nck * CK;

    const T* Ap = static_cast<const T*>(p.A);
    float A2[S], q[S], dA[S];
    float a2max = -INFINITY;
#pragma unroll
    for (int j = 0; j < S; ++j) {
        A2[j] = dv ? to_f(Ap[d * NSTATE + sg * S + j]) * LOG2E : 0.f;
        a2max = fmaxf(a2max, A2[j]);
        dA[j] = 0.f;
        q[j] = 0.f;
    }
    if (p.dh_last != nullptr && dv) {   // the I/O type, or float32 with carry32
        const int64_t off = (b * p.D + d) * NSTATE + sg * S;
#pragma unroll
        for (int j = 0; j < S; ++j)
            q[j] = p.carry32 ? static_cast<const float*>(p.dh_last)[off + j]
                             : to_f(static_cast<const T*>(p.dh_last)[off + j]);
    }
    const float Dd = dv ? to_f(static_cast<const T*>(p.Dv)[d]) : 0.f;
    float dD = 0.f;

    const int64_t boff = b * p.L * p.D + d0;
    const T* ub = static_cast<const T*>(p.u) + boff;
    const T* db = static_cast<const T*>(p.delta) + boff;
    const T* gb = static_cast<const T*>(p.dout) + boff;
    T* dub = static_cast<T*>(p.du) + boff;
    T* ddb = static_cast<T*>(p.ddelta) + boff;
    const T* Bb = static_cast<const T*>(p.Bm) + b * p.L * NSTATE;
    const T* Cb = static_cast<const T*>(p.Cm) + b * p.L * NSTATE;
    const int oidx = (chw < S) ? (sg * S + chw) : (NSTATE + sg * S + chw - S);

    for (int k = p.nck - 1; k >= 0; --k) {
        const int64_t t0 = (int64_t)k * CK;
        const int nrows = (int)min((int64_t)LT, p.L - t0);
        __syncthreads();
        load_tile<T, LT, CPB, NT>(su, ub + t0 * p.D, p.D, nrows, ncols, vec);
        load_tile<T, LT, CPB, NT>(sd, db + t0 * p.D, p.D, nrows, ncols, vec);
        load_tile<T, LT, CPB, NT>(sgy, gb + t0 * p.D, p.D, nrows, ncols, vec);
        load_tile_f32<T, LT, NSTATE, NT>(sB, Bb + t0 * NSTATE, NSTATE, nrows);
        load_tile_f32<T, LT, NSTATE, NT>(sC, Cb + t0 * NSTATE, NSTATE, nrows);
        float h0[S];
#pragma unroll
        for (int j = 0; j < S; ++j) h0[j] = 0.f;
        if (dv) {
            if (k == 0) {
                if (p.h_prev != nullptr) {
                    const int64_t off = (b * p.D + d) * NSTATE + sg * S;
#pragma unroll
                    for (int j = 0; j < S; ++j)
                        h0[j] = p.carry32 ? static_cast<const float*>(p.h_prev)[off + j]
                                          : to_f(static_cast<const T*>(p.h_prev)[off + j]);
                }
            } else {
                const float* c = p.ckpt + ((b * p.nck + k - 1) * p.D + d) * NSTATE + sg * S;
#pragma unroll
                for (int j = 0; j < S; ++j) h0[j] = c[j];
            }
        }
        __syncthreads();

        // Recompute the chunk's states (rows past L are zero: state unchanged).
        float hc[LT][S];
        {
            float h[S];
#pragma unroll
            for (int j = 0; j < S; ++j) h[j] = h0[j];
#pragma unroll
            for (int i = 0; i < LT; ++i) {
                const float dt = to_f(sd[i][cib]);
                const float du = dt * to_f(su[i][cib]);
                const bool clampy = dt * a2max > ARG2_HI;
#pragma unroll
                for (int j = 0; j < S; ++j) {
                    const float x = dt * A2[j];
                    const float a = ex2(clampy ? fminf(x, ARG2_HI) : x);
                    h[j] = fmaf(a, h[j], du * sB[i][sg * S + j]);
                    hc[i][j] = h[j];
                }
            }
        }

        // Adjoint pass through the chunk.
#pragma unroll
        for (int i = LT - 1; i >= 0; --i) {
            const float dt = to_f(sd[i][cib]);
            const float uu = to_f(su[i][cib]);
            const float gy = to_f(sgy[i][cib]);
            const float du = dt * uu;
            const bool clampy = dt * a2max > ARG2_HI;
            float s1 = 0.f, s2 = 0.f;
            float v[2 * S];
#pragma unroll
            for (int j = 0; j < S; ++j) {
                const int n = sg * S + j;
                const float x = dt * A2[j];
                const float a = ex2(clampy ? fminf(x, ARG2_HI) : x);
                const float g = fmaf(gy, sC[i][n], q[j]);
                const float hprev = (i > 0) ? hc[i - 1][j] : h0[j];
                const float pp = g * (a * hprev);
                s1 = fmaf(A2[j], pp, s1);
                dA[j] = fmaf(dt, pp, dA[j]);
                s2 = fmaf(g, sB[i][n], s2);
                v[j] = g * du;
                v[S + j] = gy * hc[i][j];
                q[j] = a * g;
            }
#pragma unroll
            for (int o = P / 2; o > 0; o >>= 1) {
                s1 += __shfl_xor_sync(FULL, s1, o);
                s2 += __shfl_xor_sync(FULL, s2, o);
            }
            if (sg == 0) {
                sdu[i][cib] = from_f<T>(fmaf(gy, Dd, dt * s2));
                sdd[i][cib] = from_f<T>(fmaf(uu, s2, s1 * LN2));
            }
            dD = fmaf(gy, uu, dD);
            const float r = reduce_scatter_channels<S, P>(v, chw);
            sred[warp][i][oidx] = r;
        }
        __syncthreads();
        store_tile<T, LT, CPB, NT>(dub + t0 * p.D, sdu, p.D, nrows, ncols, vec);
        store_tile<T, LT, CPB, NT>(ddb + t0 * p.D, sdd, p.D, nrows, ncols, vec);
        float* wb = p.ws_bc + (((int64_t)blockIdx.x * p.B + b) * Lp + t0) * (2 * NSTATE);
        for (int idx = threadIdx.x; idx < LT * 2 * NSTATE; idx += NT) {
            const int i = idx / (2 * NSTATE), vv = idx % (2 * NSTATE);
            float s = 0.f;
#pragma unroll
            for (int w = 0; w < NW; ++w) s += sred[w][i][vv];
            wb[idx] = s;
        }
    }

    if (!dv) return;
    float* wa = p.ws_a + (b * p.D + d) * NSTATE + sg * S;
#pragma unroll
    for (int j = 0; j < S; ++j) wa[j] = dA[j];
    if (sg == 0) p.ws_d[b * p.D + d] = dD;
    if (p.dh_prev != nullptr) {
        const int64_t off = (b * p.D + d) * NSTATE + sg * S;
#pragma unroll
        for (int j = 0; j < S; ++j) {
            if (p.carry32) static_cast<float*>(p.dh_prev)[off + j] = q[j];
            else static_cast<T*>(p.dh_prev)[off + j] = from_f<T>(q[j]);
        }
    }
}

// Fixed-order sums of the per-CTA / per-batch partials into dA, dB, dC, dD (dtype T).
template <typename T>
__global__ void ss_bwd_final_kernel(const BwdFinalArgs p) {
    const int64_t Lp = (int64_t)p.nck * CK;
    const int64_t n_bc = p.B * p.L * 2 * NSTATE;
    const int64_t n_a = p.D * NSTATE;
    const int64_t total = n_bc + n_a + p.D;
    T* dA = static_cast<T*>(p.dA);
    T* dB = static_cast<T*>(p.dB);
    T* dC = static_cast<T*>(p.dC);
    T* dD = static_cast<T*>(p.dD);
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        if (idx < n_bc) {
            const int64_t v = idx % (2 * NSTATE);
            const int64_t bt = idx / (2 * NSTATE);
            const int64_t b = bt / p.L, t = bt % p.L;
            float s = 0.f;
            for (int blk = 0; blk < p.nblk; ++blk)
                s += p.ws_bc[(((int64_t)blk * p.B + b) * Lp + t) * (2 * NSTATE) + v];
            if (v < NSTATE) dB[bt * NSTATE + v] = from_f<T>(s);
            else dC[bt * NSTATE + v - NSTATE] = from_f<T>(s);
        } else if (idx < n_bc + n_a) {
            const int64_t i = idx - n_bc;
            float s = 0.f;
            for (int64_t b = 0; b < p.B; ++b) s += p.ws_a[b * n_a + i];
            dA[i] = from_f<T>(s);
        } else {
            const int64_t i = idx - n_bc - n_a;
            float s = 0.f;
            for (int64_t b = 0; b < p.B; ++b) s += p.ws_d[b * p.D + i];
            dD[i] = from_f<T>(s);
        }
    }
}

int bwd_channels_per_block(int dtype) {
    (void)dtype;
    return BWD_NW * (32 / (NSTATE / BWD_S));
}

cudaError_t launch_bwd(const BwdArgs& a, int dtype, cudaStream_t s) {
    constexpr int CPB = BWD_NW * (32 / (NSTATE / BWD_S));
    dim3 grid((unsigned)((a.D + CPB - 1) / CPB), (unsigned)a.B, 1);
    if (dtype == 2) ss_bwd_kernel<__nv_bfloat16, BWD_S, BWD_NW><<<grid, BWD_NW * 32, 0, s>>>(a);
    else if (dtype == 1) ss_bwd_kernel<__half, BWD_S, BWD_NW><<<grid, BWD_NW * 32, 0, s>>>(a);
    else ss_bwd_kernel<float, BWD_S, BWD_NW><<<grid, BWD_NW * 32, 0, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_bwd_final(const BwdFinalArgs& a, int dtype, cudaStream_t s) {
    const int64_t total = a.B * a.L * 2 * NSTATE + a.D * NSTATE + a.D;
    const int threads = 256;
    int64_t blocks = (total + threads - 1) / threads;
    if (blocks > 148 * 8) blocks = 148 * 8;
    if (blocks < 1) blocks = 1;
    if (dtype == 2) ss_bwd_final_kernel<__nv_bfloat16><<<(unsigned)blocks, threads, 0, s>>>(a);
    else if (dtype == 1) ss_bwd_final_kernel<__half><<<(unsigned)blocks, threads, 0, s>>>(a);
    else ss_bwd_final_kernel<float><<<(unsigned)blocks, threads, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace mwc
