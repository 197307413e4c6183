// Adjoint state at the start of a time range of the selective scan (mwc_ss_adjoint_seq), from
// the adjoint q_in entering at the range end and the range's output gradient dout. The
// sequence-sharded backward needs only this on its first pass (the adjoint a range hands to
// the ranges before it), not the gradients of a full reverse scan:
//   q_L = q_in,  q_t = a_t (dout_t C_t + q_{t+1}),  q_out = q_0,  a_t = exp(min(delta_t A, 88))
// the reverse-scan recurrence of the backward (mamba_windows_cuda/mamba_cuda.py:703-742),
// with the clamped factor the backward kernels use.
//
// Two kernels. adjoint_chunk_kernel: per (batch row, channel, chunk of AJS_CH steps) one
// thread walks the chunk backwards for the channel's 16 states from a zero adjoint, giving
// the chunk's local adjoint R_c and the exponent sum E_c of its decay P_c = prod_t a_t
// (base 2). adjoint_fold_kernel: per (row, channel, state) the chunks fold from the end,
// q = R_c + 2^{E_c} q. One ex2 per (step, channel, state), as in the forward's state-only
// pass; delta and dout are read once, consecutive threads taking consecutive channels, and
// the chunk's C rows are staged once per block in shared memory as float32.
#include "mwc_b200.h"
#include "mwc_device.cuh"
#include "mwc_internal.h"

namespace mwc {

constexpr int AJS_CH = 256;    // steps per chunk
constexpr int AJS_NT = 128;    // threads (channels) per block

template <typename T>
__global__ void __launch_bounds__(AJS_NT) adjoint_chunk_kernel(
    const T* __restrict__ delta, const T* __restrict__ A, const T* __restrict__ Cm, const T* __restrict__ dout,
    float* __restrict__ R, float* __restrict__ E, int64_t L, int64_t D, int nchunks) {
    __shared__ __align__(16) float sC[AJS_CH][NSTATE];
    const int64_t d = (int64_t)blockIdx.x * AJS_NT + threadIdx.x;
    const int c = blockIdx.y;
    const int64_t b = blockIdx.z;
    const int64_t t0 = (int64_t)c * AJS_CH;
    const int n_steps = (int)min((int64_t)AJS_CH, L - t0);
    const T* Cb = Cm + (b * L + t0) * NSTATE;
    for (int i = threadIdx.x; i < n_steps * NSTATE; i += AJS_NT) (&sC[0][0])[i] = to_f(Cb[i]);
    __syncthreads();
    if (d >= D) return;

    float2 A2[NSTATE / 2], q[NSTATE / 2], e[NSTATE / 2];
#pragma unroll
    for (int j = 0; j < NSTATE / 2; ++j) {
        A2[j] = make_float2(to_f(A[d * NSTATE + 2 * j]) * LOG2E, to_f(A[d * NSTATE + 2 * j + 1]) * LOG2E);
        q[j] = make_float2(0.f, 0.f);
        e[j] = make_float2(0.f, 0.f);
    }
    const T* db = delta + (b * L + t0) * D + d;
    const T* gb = dout + (b * L + t0) * D + d;
    for (int i = n_steps - 1; i >= 0; --i) {
        const float dt = to_f(db[(int64_t)i * D]);
        const float g = to_f(gb[(int64_t)i * D]);
        const float2 dt2 = make_float2(dt, dt), g2 = make_float2(g, g);
        const float4* C4 = reinterpret_cast<const float4*>(&sC[i][0]);
#pragma unroll
        for (int j4 = 0; j4 < NSTATE / 4; ++j4) {
            const float4 cv = C4[j4];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int j = 2 * j4 + h;
                const float2 x = __fmul2_rn(dt2, A2[j]);
                const float2 xc = make_float2(fminf(x.x, ARG2_HI), fminf(x.y, ARG2_HI));
                const float2 a = make_float2(ex2(xc.x), ex2(xc.y));
                const float2 cc = h == 0 ? make_float2(cv.x, cv.y) : make_float2(cv.z, cv.w);
                q[j] = __fmul2_rn(a, __ffma2_rn(g2, cc, q[j]));
                e[j] = __fadd2_rn(e[j], xc);
            }
        }
    }
    const int64_t o = ((b * nchunks + c) * D + d) * NSTATE;
#pragma unroll
    for (int j4 = 0; j4 < NSTATE / 4; ++j4) {
        reinterpret_cast<float4*>(R + o)[j4] = make_float4(q[2 * j4].x, q[2 * j4].y, q[2 * j4 + 1].x, q[2 * j4 + 1].y);
        reinterpret_cast<float4*>(E + o)[j4] = make_float4(e[2 * j4].x, e[2 * j4].y, e[2 * j4 + 1].x, e[2 * j4 + 1].y);
    }
}

__global__ void __launch_bounds__(256) adjoint_fold_kernel(const float* __restrict__ R, const float* __restrict__ E,
                                                           const float* __restrict__ q_in, float* __restrict__ q_out,
                                                           int64_t B, int64_t D, int nchunks) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;   // (b, d, n)
    const int64_t per_row = D * NSTATE;
    if (i >= B * per_row) return;
    const int64_t b = i / per_row, dn = i % per_row;
    float q = q_in != nullptr ? q_in[i] : 0.f;
    for (int c = nchunks - 1; c >= 0; --c) {
        const int64_t o = (b * nchunks + c) * per_row + dn;
        q = fmaf(ex2(E[o]), q, R[o]);
    }
    q_out[i] = q;
}

int64_t adjoint_seq_chunks(int64_t L) { return (L + AJS_CH - 1) / AJS_CH; }

template <typename T>
static cudaError_t launch_adjoint_t(const void* delta, const void* A, const void* Cm, const void* dout,
                                    const float* q_in, float* q_out, float* ws, int64_t B, int64_t L,
                                    int64_t D, cudaStream_t s) {
    const int nch = (int)adjoint_seq_chunks(L);
    float* R = ws;
    float* E = ws + B * nch * D * NSTATE;
    const dim3 grid((unsigned)((D + AJS_NT - 1) / AJS_NT), (unsigned)nch, (unsigned)B);
    adjoint_chunk_kernel<T><<<grid, AJS_NT, 0, s>>>(static_cast<const T*>(delta), static_cast<const T*>(A),
                                                    static_cast<const T*>(Cm), static_cast<const T*>(dout), R,
                                                    E, L, D, nch);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const int64_t n = B * D * NSTATE;
    adjoint_fold_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(R, E, q_in, q_out, B, D, nch);
    return cudaGetLastError();
}

cudaError_t launch_adjoint_seq(const void* delta, const void* A, const void* Cm, const void* dout,
                               const float* q_in, float* q_out, float* ws, int64_t B, int64_t L, int64_t D,
                               int dtype, cudaStream_t s) {
    switch (dtype) {
        case MWC_F32: return launch_adjoint_t<float>(delta, A, Cm, dout, q_in, q_out, ws, B, L, D, s);
        case MWC_F16: return launch_adjoint_t<__half>(delta, A, Cm, dout, q_in, q_out, ws, B, L, D, s);
        default: return launch_adjoint_t<__nv_bfloat16>(delta, A, Cm, dout, q_in, q_out, ws, B, L, D, s);
    }
}

}  // namespace mwc
