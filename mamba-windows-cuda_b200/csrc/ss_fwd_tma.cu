// Persistent, TMA-pipelined forward selective scan for sm_100a.
//
// Work decomposition: a "chain" is one batch row x 128 channels over all of L; each chain
// is cut into K time segments. Units (segment k of chain c) are taken from a global
// atomic counter in segment-major order by one persistent CTA per SM, so the B*D/128
// chains spread evenly over the SMs even when there are only slightly more chains than SMs
// (config 3: 160 chains on 148 SMs). Segment k starts from the state segment k-1
// published (release/acquire flag); because segments are taken in order, the publisher
// is always a CTA that is already running, so the wait always ends (and is bounded).
//
// Per CTA: 4 warps, thread = channel, its 16 states in registers (8 float2 pairs updated
// with packed FFMA2). Tiles of 32 steps of u / delta (32 x 128) and of B / C (32 x 16)
// arrive by TMA (cp.async.bulk.tensor) into a 3-stage mbarrier ring that runs ahead
// across unit boundaries; y leaves through a double-buffered TMA store.
#include "mwc_device.cuh"
#include "mwc_internal.h"
#include "mwc_tma.cuh"

#include <cudaTypedefs.h>

#include <algorithm>

namespace mwc {

constexpr int PF_LT = 32;
constexpr int PF_CPB = 128;
constexpr int PF_NT = 256;   // 8 warps: two warps per SM sub-partition
constexpr int PF_ST = 3;
#ifndef MWC_FWD_MIN_SEG_TILES
#define MWC_FWD_MIN_SEG_TILES 2   // shortest segment (in 32-step tiles) the planner may pick
#endif

template <typename T>
struct __align__(128) PFwdSmem {
    T u[PF_ST][PF_LT][PF_CPB];
    T d[PF_ST][PF_LT][PF_CPB];
    T Bt[PF_ST][PF_LT][NSTATE];
    T Ct[PF_ST][PF_LT][NSTATE];
    T y[2][PF_LT][PF_CPB];                 // TMA store staging, double buffered
    float py[2][PF_LT][PF_CPB];            // partial <C, h> of the two state halves
    float Bf[PF_LT][NSTATE];               // float32 copies of B / C (fp16 inputs)
    float Cf[PF_LT][NSTATE];
    float Ds[PF_CPB];                      // D of the current unit's channels
    uint64_t full[PF_ST];
    int unit[PF_ST];
    int tile[PF_ST];
};

// Thread layout: tid = half * 128 + channel; half 0 holds states 0-7 of its channel,
// half 1 states 8-15 (4 float2 pairs each, packed FFMA2). Warps w and w + 4 share the
// same 32 channels, so every SM sub-partition runs two warps.
template <typename T>
__global__ void __launch_bounds__(PF_NT, 1) ss_fwd_persistent_kernel(const __grid_constant__ PFwdArgs p) {
    // Direct cast (no integer round trip): accesses stay in the shared address space.
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    PFwdSmem<T>& s = *reinterpret_cast<PFwdSmem<T>*>(smem_raw);
    if ((smem_u32(smem_raw) & 127u) != 0u) {  // TMA destinations need 128-byte alignment
        if (threadIdx.x == 0) atomicCAS(p.err, 0, ERR_SMEM_ALIGN);
        return;
    }
    const int tid = threadIdx.x;
    const int ch = tid & (PF_CPB - 1);
    const int half = tid >> 7;
    const int n0 = half * 8;               // first state of this thread
    const int total = p.nchains * p.K;
    constexpr bool HALF = sizeof(T) == 2;
    const unsigned stage_bytes =
        (unsigned)((2 * PF_LT * PF_CPB + (p.has_out ? 2 : 1) * PF_LT * NSTATE) * sizeof(T));

    // ---- producer (thread 0): unit queue + TMA issue --------------------------------
    int pu = -1, ptile = 0, ptiles = 0;
    bool pdone = false;
    auto unit_tiles = [&](int k) { return min(p.seg_tiles, p.ntiles - k * p.seg_tiles); };
    auto issue = [&](int st) {
        if (!pdone && (pu < 0 || ptile == ptiles)) {
            pu = atomicAdd(p.counter, 1);
            if (pu >= total) pdone = true;
            ptile = 0;
            if (!pdone) ptiles = unit_tiles(pu / p.nchains);
        }
        if (pdone) {
            s.unit[st] = -1;
            return;
        }
        const int c = pu % p.nchains, k = pu / p.nchains;
        const int b = c / p.nblk, blk = c % p.nblk;
        const int t0 = (k * p.seg_tiles + ptile) * PF_LT;
        s.unit[st] = pu;
        s.tile[st] = ptile;
        mbar_expect_tx(&s.full[st], stage_bytes);
        tma_load_3d(&s.u[st][0][0], &p.tm_u, &s.full[st], blk * PF_CPB, t0, b);
        tma_load_3d(&s.d[st][0][0], &p.tm_d, &s.full[st], blk * PF_CPB, t0, b);
        tma_load_3d(&s.Bt[st][0][0], &p.tm_B, &s.full[st], 0, t0, b);
        if (p.has_out) tma_load_3d(&s.Ct[st][0][0], &p.tm_C, &s.full[st], 0, t0, b);
        ++ptile;
    };

    if (tid == 0) {
        for (int st = 0; st < PF_ST; ++st) mbar_init(&s.full[st], 1);
        fence_mbar_init();
        prefetch_tmap(&p.tm_u);
        prefetch_tmap(&p.tm_d);
        prefetch_tmap(&p.tm_B);
        prefetch_tmap(&p.tm_C);
        prefetch_tmap(&p.tm_y);
        for (int st = 0; st < PF_ST; ++st) issue(st);
    }
    __syncthreads();

    const T* Ap = static_cast<const T*>(p.A);
    const T* Dp = static_cast<const T*>(p.Dv);
    float2 A2v[4], h2[4];
    float sumd = 0.f;
    int64_t d = 0;
    bool dv = false;

    for (int it = 0;; ++it) {
        const int st = it % PF_ST;
        const unsigned phase = (unsigned)(it / PF_ST) & 1u;
        const int unit = s.unit[st];
        if (unit < 0) break;
        const int tile = s.tile[st];
        const int c = unit % p.nchains, k = unit / p.nchains;
        const int b = c / p.nblk, blk = c % p.nblk;
        const int t0 = (k * p.seg_tiles + tile) * PF_LT;
        const bool last = tile == unit_tiles(k) - 1;

        if (tile == 0) {  // unit start: parameters and incoming state
            d = (int64_t)blk * PF_CPB + ch;
            dv = d < p.D;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                A2v[j].x = dv ? to_f(Ap[d * NSTATE + n0 + 2 * j]) * LOG2E : 0.f;
                A2v[j].y = dv ? to_f(Ap[d * NSTATE + n0 + 2 * j + 1]) * LOG2E : 0.f;
            }
            if (half == 0) s.Ds[ch] = dv ? to_f(Dp[d]) : 0.f;
            if (k == 0) {
                sumd = 0.f;
#pragma unroll
                for (int j = 0; j < 4; ++j) h2[j] = make_float2(0.f, 0.f);
                if (p.h_prev != nullptr && dv) {
                    const T* hp = static_cast<const T*>(p.h_prev) + ((int64_t)b * p.D + d) * NSTATE + n0;
#pragma unroll
                    for (int j = 0; j < 4; ++j) h2[j] = make_float2(to_f(hp[2 * j]), to_f(hp[2 * j + 1]));
                }
            } else {
                if (tid == 0) flag_wait(&p.flags[c * p.K + k - 1], 1, p.err);
                __syncthreads();
                const float* hs = p.hand + ((int64_t)(c * p.K + k - 1) * PF_CPB + ch) * (NSTATE + 1);
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    h2[j] = make_float2(__ldcg(hs + n0 + 2 * j), __ldcg(hs + n0 + 2 * j + 1));
                sumd = __ldcg(hs + NSTATE);
            }
        }

        mbar_wait(&s.full[st], phase, p.err);
        const float* Bf;
        const float* Cf;
        if constexpr (HALF) {
            for (int idx = tid; idx < PF_LT * NSTATE; idx += PF_NT) {
                (&s.Bf[0][0])[idx] = to_f((&s.Bt[st][0][0])[idx]);
                if (p.has_out) (&s.Cf[0][0])[idx] = to_f((&s.Ct[st][0][0])[idx]);
            }
            __syncthreads();
            Bf = &s.Bf[0][0];
            Cf = &s.Cf[0][0];
        } else {
            Bf = reinterpret_cast<const float*>(&s.Bt[st][0][0]);
            Cf = reinterpret_cast<const float*>(&s.Ct[st][0][0]);
        }

        // Blocks of 8 steps: the block's shared-memory reads precede its stores, and the
        // exponent clamp of safe_exp is a branch-free min per state, so the exponentials
        // of later steps overlap the FMAs of earlier ones.
#pragma unroll 1
        for (int i0 = 0; i0 < PF_LT; i0 += 8) {
            float dtv[8], uv[8], yv[8];
#pragma unroll
            for (int r = 0; r < 8; ++r) {
                dtv[r] = to_f(s.d[st][i0 + r][ch]);
                uv[r] = to_f(s.u[st][i0 + r][ch]);
            }
#pragma unroll
            for (int r = 0; r < 8; ++r) {
                const float dt = dtv[r];
                sumd += dt;
                const float2 dt2 = make_float2(dt, dt);
                const float2 du2 = make_float2(dt * uv[r], dt * uv[r]);
                float2 a2[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float2 x = __fmul2_rn(dt2, A2v[j]);
                    a2[j] = make_float2(ex2(fminf(x.x, ARG2_HI)), ex2(fminf(x.y, ARG2_HI)));
                }
                const float4* Bq = reinterpret_cast<const float4*>(Bf + (i0 + r) * NSTATE + n0);
                const float4* Cq = reinterpret_cast<const float4*>(Cf + (i0 + r) * NSTATE + n0);
                float2 yq[2];
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    const float4 bq = Bq[q];
                    const float4 cq = Cq[q];
                    h2[2 * q] = __ffma2_rn(a2[2 * q], h2[2 * q], __fmul2_rn(du2, make_float2(bq.x, bq.y)));
                    h2[2 * q + 1] =
                        __ffma2_rn(a2[2 * q + 1], h2[2 * q + 1], __fmul2_rn(du2, make_float2(bq.z, bq.w)));
                    yq[q] = __fmul2_rn(make_float2(cq.x, cq.y), h2[2 * q]);
                    yq[q] = __ffma2_rn(make_float2(cq.z, cq.w), h2[2 * q + 1], yq[q]);
                }
                const float2 y2 = __fadd2_rn(yq[0], yq[1]);
                yv[r] = y2.x + y2.y;
            }
#pragma unroll
            for (int r = 0; r < 8; ++r) s.py[half][i0 + r][ch] = yv[r];
            if ((i0 + 8) % CK == 0 && p.ckpt != nullptr) {
                const int64_t kk = (int64_t)(t0 + i0 + 8) / CK - 1;
                if (kk < p.nck && dv) {
                    float4* cp = reinterpret_cast<float4*>(
                        p.ckpt + (((int64_t)b * p.nck + kk) * p.D + d) * NSTATE + n0);
                    cp[0] = make_float4(h2[0].x, h2[0].y, h2[1].x, h2[1].y);
                    cp[1] = make_float4(h2[2].x, h2[2].y, h2[3].x, h2[3].y);
                }
            }
        }

        if (last) {
            if (k < p.K - 1) {
                float* hs = p.hand + ((int64_t)(c * p.K + k) * PF_CPB + ch) * (NSTATE + 1);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    hs[n0 + 2 * j] = h2[j].x;
                    hs[n0 + 2 * j + 1] = h2[j].y;
                }
                if (half == 0) hs[NSTATE] = sumd;
                __threadfence();
            } else if (dv) {
                if (p.h_last != nullptr) {
                    T* hl = static_cast<T*>(p.h_last) + ((int64_t)b * p.D + d) * NSTATE + n0;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        hl[2 * j] = from_f<T>(h2[j].x);
                        hl[2 * j + 1] = from_f<T>(h2[j].y);
                    }
                }
                if (p.decay != nullptr) {
                    float* dc = p.decay + ((int64_t)b * p.D + d) * NSTATE + n0;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        dc[2 * j] = ex2(fminf(A2v[j].x * sumd, ARG2_HI));
                        dc[2 * j + 1] = ex2(fminf(A2v[j].y * sumd, ARG2_HI));
                    }
                }
            }
        }

        // y = partial(states 0-7) + partial(states 8-15) + D u, staged for the TMA store.
        // The staging buffer of this tile was last read by the store of tile it-2.
        if (tid == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
        __syncthreads();
        if (p.has_out) {
            T (*yb)[PF_CPB] = s.y[it & 1];
#pragma unroll
            for (int r = 0; r < (PF_LT * PF_CPB) / (4 * PF_NT); ++r) {
                const int idx = (tid + r * PF_NT) * 4;
                const int i = idx / PF_CPB, cc = idx % PF_CPB;
                const float4 p0 = *reinterpret_cast<const float4*>(&s.py[0][i][cc]);
                const float4 p1 = *reinterpret_cast<const float4*>(&s.py[1][i][cc]);
                const float4 dd = *reinterpret_cast<const float4*>(&s.Ds[cc]);
                yb[i][cc + 0] = from_f<T>(fmaf(dd.x, to_f(s.u[st][i][cc + 0]), p0.x + p1.x));
                yb[i][cc + 1] = from_f<T>(fmaf(dd.y, to_f(s.u[st][i][cc + 1]), p0.y + p1.y));
                yb[i][cc + 2] = from_f<T>(fmaf(dd.z, to_f(s.u[st][i][cc + 2]), p0.z + p1.z));
                yb[i][cc + 3] = from_f<T>(fmaf(dd.w, to_f(s.u[st][i][cc + 3]), p0.w + p1.w));
            }
        }
        fence_proxy_async();
        __syncthreads();
        if (tid == 0) {
            if (p.has_out) {
                tma_store_3d(&p.tm_y, &s.y[it & 1][0][0], blk * PF_CPB, t0, b);
                bulk_commit();
            }
            if (last && k < p.K - 1) flag_release(&p.flags[c * p.K + k], 1);
            issue(st);
        }
    }
    if (tid == 0) bulk_wait0();
}

// ---------------------------------------------------------------------------- host side

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (fn == nullptr) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
    return fn;
}

// 3-D tiled map over a contiguous (outer, mid, inner) = (B, L, W) tensor, box (bw, bl, 1).
bool make_tmap_3d(CUtensorMap* map, const void* base, int dtype, int64_t W, int64_t L,
                  int64_t B, int bw, int bl) {
    auto fn = encode_fn();
    if (fn == nullptr) return false;
    const size_t es = dtype == 1 ? 2 : 4;
    cuuint64_t dims[3] = {(cuuint64_t)W, (cuuint64_t)L, (cuuint64_t)B};
    cuuint64_t strides[2] = {(cuuint64_t)(W * es), (cuuint64_t)(W * L * es)};
    cuuint32_t box[3] = {(cuuint32_t)bw, (cuuint32_t)bl, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, dtype == 1 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                    3, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

PersistPlan plan_persistent(int64_t B, int64_t L, int64_t D, int num_sms) {
    PersistPlan pl{};
    pl.nblk = (int)((D + PF_CPB - 1) / PF_CPB);
    pl.nchains = (int)(B * pl.nblk);
    pl.ntiles = (int)((L + PF_LT - 1) / PF_LT);
    pl.ok = pl.nchains >= num_sms;
    int best_k = 1;
    double best = -1.0;
    for (int K = 1; K <= pl.ntiles; ++K) {
        const int seg = (pl.ntiles + K - 1) / K;
        const int keff = (pl.ntiles + seg - 1) / seg;
        if (keff != K) continue;
        if (K > 1 && seg < MWC_FWD_MIN_SEG_TILES) break;
        const int64_t U = (int64_t)pl.nchains * K;
        const int64_t G = std::min<int64_t>(num_sms, U);
        const int64_t waves = (U + G - 1) / G;
        const double eff = (double)U / (double)(G * waves);
        if (eff > best + 0.01) {
            best = eff;
            best_k = K;
        }
    }
    pl.K = best_k;
    pl.seg_tiles = (pl.ntiles + best_k - 1) / best_k;
    pl.grid = (int)std::min<int64_t>(num_sms, (int64_t)pl.nchains * pl.K);
    return pl;
}

int64_t persistent_ws_bytes(const PersistPlan& pl) {
    const int64_t units = (int64_t)pl.nchains * pl.K;
    const int64_t hdr = ((16 + units * 4) + 255) / 256 * 256;
    return hdr + units * PF_CPB * (NSTATE + 1) * 4;
}

int64_t persistent_ws_header(const PersistPlan& pl) {
    const int64_t units = (int64_t)pl.nchains * pl.K;
    return ((16 + units * 4) + 255) / 256 * 256;
}

template <typename T>
static cudaError_t launch_pf(const PFwdArgs& a, int grid, cudaStream_t s) {
    const size_t smem = sizeof(PFwdSmem<T>);
    cudaError_t e = cudaFuncSetAttribute(ss_fwd_persistent_kernel<T>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    ss_fwd_persistent_kernel<T><<<grid, PF_NT, smem, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_fwd_persistent(PFwdArgs& a, const PersistPlan& pl, int dtype, void* ws,
                                  cudaStream_t s) {
    char* w = static_cast<char*>(ws);
    a.counter = reinterpret_cast<int*>(w);
    a.err = reinterpret_cast<int*>(w + 4);
    a.flags = reinterpret_cast<int*>(w + 16);
    a.hand = reinterpret_cast<float*>(w + persistent_ws_header(pl));
    a.nblk = pl.nblk;
    a.nchains = pl.nchains;
    a.K = pl.K;
    a.seg_tiles = pl.seg_tiles;
    a.ntiles = pl.ntiles;
    cudaError_t e = cudaMemsetAsync(ws, 0, (size_t)persistent_ws_header(pl), s);
    if (e != cudaSuccess) return e;
    return dtype == 1 ? launch_pf<__half>(a, pl.grid, s) : launch_pf<float>(a, pl.grid, s);
}

}  // namespace mwc
