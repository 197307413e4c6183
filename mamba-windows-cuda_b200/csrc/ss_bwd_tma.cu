// Persistent, warp-specialized, TMA-pipelined backward selective scan for sm_100a.
//
// Same work decomposition as the persistent forward (chains of 128 channels of one batch
// row, cut into K time segments, taken from an atomic queue), walked in reverse: the unit
// for the last time segment of a chain starts from dh_last, every other unit starts from
// the adjoint state q its successor segment published (8 per-warp increments of a flag;
// bounded wait).
//
// Per 16-step tile (= one checkpoint chunk), processed last tile first:
//   * the producer warp brings u, delta, dout (16 x 128) and B, C (16 x 16) by TMA and
//     the float32 checkpoint state at the chunk start (128 x 16) by a 1-D bulk copy into
//     a 2-stage mbarrier ring;
//   * 8 compute warps recompute the chunk's states forward into a per-thread shared-memory
//     cache (conflict-free float4 layout), then run the adjoint recurrence backwards:
//       g = dout C + q,  p = g a h_{t-1},  ddelta = ln2 <A2, p> + u <g, B>,
//       du = dout D + delta <g, B>,  dA += delta p,  q = a g,
//       dB_t = sum_d g delta u,  dC_t = sum_d dout h_t;
//   * the helper warp converts B / C to float32 (fp16 inputs), sums the 8 warps' dB / dC
//     partials of a tile in warp order into the per-block workspace, and (fp16) stores the
//     du / ddelta tiles by TMA.
// Thread layout: warp w covers channels 16w .. 16w+15; lane = (cg, sg) with cg = lane / 4
// the channel pair and sg = lane % 4 the state group (4 states): a thread owns 2 channels x
// 4 states, so the cross-channel sums of dB / dC start as in-thread FMAs and finish with a
// 3-level butterfly over the 8 channel pairs of the warp; the per-channel sums over states
// take 2 shuffle levels. Every reduction has a fixed order (butterfly, warps in order, then
// the finalize kernel over blocks / segments / batch rows in order): results are bitwise
// reproducible.
#include "mwc_device.cuh"
#include "mwc_internal.h"
#include "mwc_tma.cuh"

#include <algorithm>
#include <type_traits>

namespace mwc {

constexpr int PB_LT = CK;     // 16 steps per tile
constexpr int PB_CPB = 128;
constexpr int PB_NCW = 8;                    // compute warps
constexpr int PB_NCT = PB_NCW * 32;          // compute threads
constexpr int PB_NT = (PB_NCW + 2) * 32;     // + producer warp + helper warp
constexpr int PB_ST = 4;
// TMEM state cache: per compute thread and step, the state before the step (8 values) and
// the decay factors of the step (8 values); 16 steps x 16 columns = 256 columns per thread,
// warps w and w + 4 share a lane quarter and split the 512 columns.
constexpr uint32_t PB_TMEM_COLS = 512;
#ifndef MWC_BWD_MIN_SEG_TILES
#define MWC_BWD_MIN_SEG_TILES 4   // shortest segment (in 16-step tiles) the planner may pick
#endif

template <typename T>
struct PbCfg {
    static constexpr bool HALF = sizeof(T) == 2;
    static constexpr int RB = HALF ? 2 : 1;       // dB | dC partial buffers
    static constexpr bool STAGE_OUT = HALF;       // du / ddelta staged for TMA stores
};

template <typename T>
struct __align__(128) PBwdSmem {
    using C = PbCfg<T>;
    float h0[PB_ST][PB_CPB][NSTATE];             // checkpoint at the chunk start
    float qin[PB_ST][PB_CPB][NSTATE];            // incoming adjoint state (unit start)
    T At[PB_ST][PB_CPB][NSTATE];                 // unit parameters: A rows,
    T Dt[PB_ST][PB_CPB];                         // D
    T u[PB_ST][PB_LT][PB_CPB];
    T d[PB_ST][PB_LT][PB_CPB];
    T g[PB_ST][PB_LT][PB_CPB];
    T Bt[PB_ST][PB_LT][NSTATE];
    T Ct[PB_ST][PB_LT][NSTATE];
    T duo[C::STAGE_OUT ? 2 : 1][C::STAGE_OUT ? PB_LT : 1][C::STAGE_OUT ? PB_CPB : 8];  // du / ddelta
    T ddo[C::STAGE_OUT ? 2 : 1][C::STAGE_OUT ? PB_LT : 1][C::STAGE_OUT ? PB_CPB : 8];  // staging
    float red[C::RB][PB_NCW][PB_LT][2 * NSTATE];  // per-warp dB | dC partials of a tile
    float Bf[C::HALF ? PB_ST : 1][PB_LT][NSTATE];
    float Cf[C::HALF ? PB_ST : 1][PB_LT][NSTATE];
    uint64_t full[PB_ST], conv[PB_ST], empty[PB_ST], qfull[PB_ST];
    uint64_t redfull[C::RB], redempty[C::RB], ofull[2], oempty[2];
    int unit[PB_ST];
    int tile[PB_ST];
    int dpos[PB_ST];   // helper: 1 when no delta of the stage's tile has its sign bit set
    uint32_t tmem_base;
};

__device__ __forceinline__ void bulk_load(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void mbar_arrive_b(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

template <typename T>
__device__ __forceinline__ void load2(float (&v)[2], const T* p);
template <>
__device__ __forceinline__ void load2<float>(float (&v)[2], const float* p) {
    const float2 x = *reinterpret_cast<const float2*>(p);
    v[0] = x.x; v[1] = x.y;
}
template <>
__device__ __forceinline__ void load2<__half>(float (&v)[2], const __half* p) {
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(p));
    v[0] = a.x; v[1] = a.y;
}

template <>
__device__ __forceinline__ void load2<__nv_bfloat16>(float (&v)[2], const __nv_bfloat16* p) {
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
    v[0] = a.x; v[1] = a.y;
}

template <typename T>
__device__ __forceinline__ void load4(float (&v)[4], const T* p);
template <>
__device__ __forceinline__ void load4<float>(float (&v)[4], const float* p) {
    const float4 x = *reinterpret_cast<const float4*>(p);
    v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
}
template <>
__device__ __forceinline__ void load4<__half>(float (&v)[4], const __half* p) {
    const uint2 raw = *reinterpret_cast<const uint2*>(p);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}

template <>
__device__ __forceinline__ void load4<__nv_bfloat16>(float (&v)[4], const __nv_bfloat16* p) {
    const uint2 raw = *reinterpret_cast<const uint2*>(p);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}

template <typename T>
__device__ __forceinline__ void store2(T* p, float a, float b);
template <>
__device__ __forceinline__ void store2<float>(float* p, float a, float b) {
    *reinterpret_cast<float2*>(p) = make_float2(a, b);
}
template <>
__device__ __forceinline__ void store2<__half>(__half* p, float a, float b) {
    *reinterpret_cast<__half2*>(p) = __floats2half2_rn(a, b);
}

template <>
__device__ __forceinline__ void store2<__nv_bfloat16>(__nv_bfloat16* p, float a, float b) {
    *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(a, b);
}

template <typename T>
__device__ __forceinline__ void store4(T* p, const float (&v)[4]);
template <>
__device__ __forceinline__ void store4<float>(float* p, const float (&v)[4]) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}
template <>
__device__ __forceinline__ void store4<__half>(__half* p, const float (&v)[4]) {
    __half2 a = __floats2half2_rn(v[0], v[1]);
    __half2 b = __floats2half2_rn(v[2], v[3]);
    uint2 raw;
    raw.x = *reinterpret_cast<uint32_t*>(&a);
    raw.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = raw;
}
template <>
__device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16* p, const float (&v)[4]) {
    __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]);
    __nv_bfloat162 b = __floats2bfloat162_rn(v[2], v[3]);
    uint2 raw;
    raw.x = *reinterpret_cast<uint32_t*>(&a);
    raw.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = raw;
}

__device__ __forceinline__ float2 f2(float x) { return make_float2(x, x); }

// A (B, D, 16) state row: the I/O type, or float32 when the launch carries its states in
// float32 (the sequence-sharded backward's h_in / q_in / q_out)
template <typename T>
__device__ __forceinline__ void load_state4(float (&v)[4], const void* base, int64_t off, bool c32) {
    if (c32) load4<float>(v, static_cast<const float*>(base) + off);
    else load4<T>(v, static_cast<const T*>(base) + off);
}
template <typename T>
__device__ __forceinline__ void store_state4(void* base, int64_t off, const float (&v)[4], bool c32) {
    if (c32) store4<float>(static_cast<float*>(base) + off, v);
    else store4<T>(static_cast<T*>(base) + off, v);
}

template <typename T>
__global__ void __launch_bounds__(PB_NT, 1) ss_bwd_persistent_kernel(const __grid_constant__ PBwdArgs p) {
    // Direct cast (no integer round trip): accesses stay in the shared address space.
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    PBwdSmem<T>& s = *reinterpret_cast<PBwdSmem<T>*>(smem_raw);
    using Cfg = PbCfg<T>;
    constexpr bool HALF = Cfg::HALF;
    constexpr int RB = Cfg::RB;
    if ((smem_u32(smem_raw) & 127u) != 0u) {  // TMA destinations need 128-byte alignment
        if (threadIdx.x == 0) atomicCAS(p.err, 0, ERR_SMEM_ALIGN);
        return;
    }
    const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
    const int total = p.nchains * p.K;
    const int64_t Lp = (int64_t)p.nck * CK;

    if (tid == 0) {
        for (int i = 0; i < PB_ST; ++i) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.conv[i], 1);
            mbar_init(&s.empty[i], PB_NCW);
            mbar_init(&s.qfull[i], 1);
        }
        for (int i = 0; i < RB; ++i) {
            mbar_init(&s.redfull[i], PB_NCW);
            mbar_init(&s.redempty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s.ofull[i], PB_NCW);
            mbar_init(&s.oempty[i], 1);
        }
        fence_mbar_init();
    }
    if (w == 0) {   // one CTA per SM (shared memory > half the SM), so the allocation succeeds
        __syncwarp();   // lane 0 initialised the barriers; the allocation is warp-collective
        tmem_alloc(&s.tmem_base, PB_TMEM_COLS);
        tmem_relinquish();
    }
    tmem_fence_before_sync();
    __syncthreads();
    tmem_fence_after_sync();

    if (w == PB_NCW) {
        // ============================== producer ==============================
        if (lane != 0) return;
        prefetch_tmap(&p.tm_u);
        prefetch_tmap(&p.tm_d);
        prefetch_tmap(&p.tm_g);
        prefetch_tmap(&p.tm_B);
        prefetch_tmap(&p.tm_C);
        const unsigned tile_bytes = (unsigned)((3 * PB_LT * PB_CPB + 2 * PB_LT * NSTATE) * sizeof(T));
        int pu = -1, pcount = 0, ptiles = 0, pfirst = 0;
        for (int it = 0;; ++it) {
            const int st = it % PB_ST;
            mbar_wait(&s.empty[st], ((unsigned)(it / PB_ST) & 1u) ^ 1u, p.err);
            if (pu < 0 || pcount == ptiles) {
                pu = atomicAdd(p.counter, 1);
                if (pu >= total) {
                    s.unit[st] = -1;
                    mbar_arrive_b(&s.full[st]);
                    return;
                }
                const int k = p.K - 1 - pu / p.nchains;
                pfirst = k * p.seg_tiles;
                ptiles = min(p.seg_tiles, p.ntiles - pfirst);
                pcount = 0;
            }
            const int c = pu % p.nchains, kp = pu / p.nchains;
            const int b = c / p.nblk, blk = c % p.nblk;
            const int tix = pfirst + ptiles - 1 - pcount;
            const int t0 = tix * PB_LT;
            s.unit[st] = pu;
            s.tile[st] = pcount;
            const int nch = min(PB_CPB, p.D - blk * PB_CPB);
            const unsigned hbytes = tix > 0 ? (unsigned)(nch * NSTATE * 4) : 0u;
            const unsigned rbytes = pcount == 0 ? (unsigned)(nch * (NSTATE + 1) * sizeof(T)) : 0u;
            mbar_expect_tx(&s.full[st], tile_bytes + hbytes + rbytes);
            tma_load_3d(&s.u[st][0][0], &p.tm_u, &s.full[st], blk * PB_CPB, t0, b);
            tma_load_3d(&s.d[st][0][0], &p.tm_d, &s.full[st], blk * PB_CPB, t0, b);
            tma_load_3d(&s.g[st][0][0], &p.tm_g, &s.full[st], blk * PB_CPB, t0, b);
            const int gx = (blk * PB_CPB / p.cpg) * NSTATE;   // the block's B / C group
            tma_load_3d(&s.Bt[st][0][0], &p.tm_B, &s.full[st], gx, t0, b);
            tma_load_3d(&s.Ct[st][0][0], &p.tm_C, &s.full[st], gx, t0, b);
            if (tix > 0)
                bulk_load(&s.h0[st][0][0],
                          p.ckpt + (((int64_t)b * p.nck + tix - 1) * p.D + (int64_t)blk * PB_CPB) * NSTATE,
                          hbytes, &s.full[st]);
            if (pcount == 0) {
                bulk_load(&s.At[st][0][0], static_cast<const T*>(p.A) + (int64_t)blk * PB_CPB * NSTATE,
                          (unsigned)(nch * NSTATE * sizeof(T)), &s.full[st]);
                bulk_load(&s.Dt[st][0], static_cast<const T*>(p.Dv) + (int64_t)blk * PB_CPB,
                          (unsigned)(nch * sizeof(T)), &s.full[st]);
                if (kp > 0) {
                    // the tile is already on its way; the adjoint state of the successor
                    // segment follows on its own barrier, which the compute warps wait for
                    // only after their recompute pass (seeded: the record is already there)
                    if (p.mode == 0) flag_wait(&p.flags[c * p.K + kp - 1], PB_NCW, p.err);
                    fence_proxy_async_global();
                    mbar_expect_tx(&s.qfull[st], (unsigned)(PB_CPB * NSTATE * 4));
                    bulk_load(&s.qin[st][0][0], p.hand + (int64_t)(c * p.K + kp - 1) * PB_CPB * NSTATE,
                              (unsigned)(PB_CPB * NSTATE * 4), &s.qfull[st]);
                }
            }
            ++pcount;
        }
    }

    if (w == PB_NCW + 1) {
        // ======= helper: float32 B / C, ordered dB | dC partials, du / ddelta stores =======
        if constexpr (Cfg::STAGE_OUT) {
            prefetch_tmap(&p.tm_du);
            prefetch_tmap(&p.tm_dd);
        }
        int pb = 0, pblk = 0, pt0 = 0;
        for (int it = 0;; ++it) {
            const int st = it % PB_ST;
            mbar_wait(&s.full[st], (unsigned)(it / PB_ST) & 1u, p.err);
            const int unit = s.unit[st];
            int b = 0, blk = 0, t0 = 0;
            if (unit >= 0) {
                const int c = unit % p.nchains, kp = unit / p.nchains, k = p.K - 1 - kp;
                b = c / p.nblk;
                blk = c % p.nblk;
                const int first = k * p.seg_tiles;
                const int ntl = min(p.seg_tiles, p.ntiles - first);
                t0 = (first + ntl - 1 - s.tile[st]) * PB_LT;
                if constexpr (HALF) {
                    for (int idx = lane; idx < PB_LT * NSTATE; idx += 32) {
                        (&s.Bf[HALF ? st : 0][0][0])[idx] = to_f((&s.Bt[st][0][0])[idx]);
                        (&s.Cf[HALF ? st : 0][0][0])[idx] = to_f((&s.Ct[st][0][0])[idx]);
                    }
                }
                // safe_exp's clamp is the identity for the whole tile when no delta is
                // negative (given A <= 0): OR of the raw sign bits of the delta tile
                const uint4* dw = reinterpret_cast<const uint4*>(&s.d[st][0][0]);
                constexpr int NW4 = PB_LT * PB_CPB * (int)sizeof(T) / 16;
                constexpr uint32_t SIGN = sizeof(T) == 2 ? 0x80008000u : 0x80000000u;
                uint32_t neg = 0;
#pragma unroll 4
                for (int idx = lane; idx < NW4; idx += 32) {
                    const uint4 v = dw[idx];
                    neg |= (v.x | v.y | v.z | v.w) & SIGN;
                }
                const bool any_neg = __any_sync(FULL, neg != 0);
                if (lane == 0) s.dpos[st] = any_neg ? 0 : 1;
            } else if (lane == 0) {
                s.dpos[st] = 0;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive_b(&s.conv[st]);
            if (it > 0) {
                const int rb = (it - 1) % RB;
                mbar_wait(&s.redfull[rb], (unsigned)((it - 1) / RB) & 1u, p.err);
                // partials laid out (b, t, block, 32): the finalize reads a (b, t) row's blocks
                // as one contiguous run
                float* wb = p.ws_bc + (((int64_t)pb * Lp + pt0) * p.nblk + pblk) * (2 * NSTATE);
#pragma unroll 4
                for (int r = 0; r < (PB_LT * 2 * NSTATE) / 32; ++r) {
                    const int idx = lane + r * 32;
                    const int i = idx / (2 * NSTATE), vv = idx % (2 * NSTATE);
                    float acc = s.red[rb][0][i][vv];
#pragma unroll
                    for (int ww = 1; ww < PB_NCW; ++ww) acc += s.red[rb][ww][i][vv];
                    wb[(int64_t)i * p.nblk * (2 * NSTATE) + vv] = acc;
                }
                __syncwarp();
                if (lane == 0) mbar_arrive_b(&s.redempty[rb]);
                if constexpr (Cfg::STAGE_OUT) {
                    const int ob = (it - 1) & 1;
                    mbar_wait(&s.ofull[ob], (unsigned)((it - 1) / 2) & 1u, p.err);
                    if (lane == 0) {
                        tma_store_3d(&p.tm_du, &s.duo[ob][0][0], pblk * PB_CPB, pt0, pb);
                        tma_store_3d(&p.tm_dd, &s.ddo[ob][0][0], pblk * PB_CPB, pt0, pb);
                        bulk_commit();
                        bulk_wait_read0();
                        mbar_arrive_b(&s.oempty[ob]);
                    }
                    __syncwarp();
                }
            }
            if (unit < 0) break;
            pb = b;
            pblk = blk;
            pt0 = t0;
        }
        if (lane == 0) bulk_wait0();
        return;
    }

    // ================================ compute warps ================================
    const int cg = lane >> 2, sg = lane & 3;
    const uint32_t tcache = s.tmem_base + ((uint32_t)(32 * (w & 3)) << 16) + (uint32_t)(w >> 2) * 256u;
    const int c2 = w * 16 + cg * 2;          // first of the thread's 2 channels in the block
    float2 A2[2][2], q[2][2], dA[2][2];
    float Dd[2], dD[2];
    bool a_nonpos = true;   // warp-uniform: A <= 0, so delta >= 0 keeps every exponent <= 0
    int64_t dbase = 0;
    unsigned qphase = 0;    // bit st: parity of the next wait on qfull[st]

    for (int it = 0;; ++it) {
        const int st = it % PB_ST;
        mbar_wait(&s.full[st], (unsigned)(it / PB_ST) & 1u, p.err);
        mbar_wait(&s.conv[st], (unsigned)(it / PB_ST) & 1u, p.err);
        const int unit = s.unit[st];
        if (unit < 0) break;

        const int pc = s.tile[st];
        const int c = unit % p.nchains, kp = unit / p.nchains, k = p.K - 1 - kp;
        const int b = c / p.nblk, blk = c % p.nblk;
        const int first = k * p.seg_tiles;
        const int ntl = min(p.seg_tiles, p.ntiles - first);
        const int tix = first + ntl - 1 - pc;
        const int t0 = tix * PB_LT;
        const bool unit_end = pc == ntl - 1;
        bool dvc[2];
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) dvc[cc] = (int64_t)blk * PB_CPB + c2 + cc < p.D;

        if (pc == 0) {  // unit start
            dbase = (int64_t)blk * PB_CPB + c2;
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
                float a4[4] = {0.f, 0.f, 0.f, 0.f};
                if (dvc[cc]) load4<T>(a4, &s.At[st][c2 + cc][4 * sg]);
                A2[cc][0] = make_float2(a4[0] * LOG2E, a4[1] * LOG2E);
                A2[cc][1] = make_float2(a4[2] * LOG2E, a4[3] * LOG2E);
                Dd[cc] = dvc[cc] ? to_f(s.Dt[st][c2 + cc]) : 0.f;
                dD[cc] = 0.f;
                dA[cc][0] = dA[cc][1] = make_float2(0.f, 0.f);
            }
            a_nonpos = __all_sync(FULL, A2[0][0].x <= 0.f && A2[0][0].y <= 0.f && A2[0][1].x <= 0.f &&
                                            A2[0][1].y <= 0.f && A2[1][0].x <= 0.f && A2[1][0].y <= 0.f &&
                                            A2[1][1].x <= 0.f && A2[1][1].y <= 0.f);
            if (kp == 0) {
#pragma unroll
                for (int cc = 0; cc < 2; ++cc) {
                    float g4[4] = {0.f, 0.f, 0.f, 0.f};
                    if (p.dh_last != nullptr && dvc[cc])
                        load_state4<T>(g4, p.dh_last, ((int64_t)b * p.D + dbase + cc) * NSTATE + 4 * sg,
                                       p.carry32 != 0);
                    q[cc][0] = make_float2(g4[0], g4[1]);
                    q[cc][1] = make_float2(g4[2], g4[3]);
                }
            }
            // otherwise q arrives on qfull[st], read before the adjoint pass
        }

        // tcgen05 loads / stores are warp-collective (.sync.aligned): reconverge the lanes,
        // which leave the barrier spin loops and the divergent unit-boundary code separately
        __syncwarp();
        const float* Bf = HALF ? &s.Bf[HALF ? st : 0][0][0] : reinterpret_cast<const float*>(&s.Bt[st][0][0]);
        const float* Cf = HALF ? &s.Cf[HALF ? st : 0][0][0] : reinterpret_cast<const float*>(&s.Ct[st][0][0]);

        // state at the chunk start (channels past D stay zero)
        float2 h[2][2];
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (dvc[cc]) {
                if (tix > 0) {
                    v = *reinterpret_cast<const float4*>(&s.h0[st][c2 + cc][4 * sg]);
                } else if (p.h_prev != nullptr) {
                    float hp4[4];
                    load_state4<T>(hp4, p.h_prev, ((int64_t)b * p.D + dbase + cc) * NSTATE + 4 * sg,
                                   p.carry32 != 0);
                    v = make_float4(hp4[0], hp4[1], hp4[2], hp4[3]);
                }
            }
            h[cc][0] = make_float2(v.x, v.y);
            h[cc][1] = make_float2(v.z, v.w);
        }

        // ---- recompute: TMEM column block i = (state before step i, decay factors of step i);
        //      h ends as the state after the last step (blocks of 4 steps: loads, then the
        //      serial updates) ----
        __syncwarp();   // the chunk-start loads above depend on the channel's lane
        // safe_exp's clamp is the identity when every exponent is <= 0: A <= 0 for the unit
        // and no negative delta in the tile (uniform per tile)
        // (each copy of the recompute loop below is branch-free)
        auto recompute = [&](auto clamp_tag) {
            constexpr bool CLAMP = decltype(clamp_tag)::value;
            // two 4-step blocks per iteration: the second block's loads and exponentials
            // overlap the first block's serial updates (fp16: 168 registers, no spills).
            // 168 is the ceiling (the sub-partitions with 3 of the 10 warps hold 3 x 32 x 168
            // of their 16,384 registers); bfloat16 spilled 116 bytes with two blocks and runs
            // 3% faster with one (158 registers, no spills)
            constexpr int RU = std::is_same<T, __nv_bfloat16>::value ? 1 : 2;
#pragma unroll RU
        for (int i0 = 0; i0 < PB_LT; i0 += 4) {
            float dt[4][2], uu[4][2];
            float4 B4[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                load2<T>(dt[r], &s.d[st][i0 + r][c2]);
                load2<T>(uu[r], &s.u[st][i0 + r][c2]);
                B4[r] = *reinterpret_cast<const float4*>(Bf + (i0 + r) * NSTATE + 4 * sg);
            }
            float2 x[4][2][2];
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int cc = 0; cc < 2; ++cc) {
                    x[r][cc][0] = __fmul2_rn(f2(dt[r][cc]), A2[cc][0]);
                    x[r][cc][1] = __fmul2_rn(f2(dt[r][cc]), A2[cc][1]);
                }
            if constexpr (CLAMP) {
#pragma unroll
                for (int r = 0; r < 4; ++r)
#pragma unroll
                    for (int cc = 0; cc < 2; ++cc)
#pragma unroll
                        for (int pr = 0; pr < 2; ++pr)
                            x[r][cc][pr] = make_float2(fminf(x[r][cc][pr].x, ARG2_HI),
                                                       fminf(x[r][cc][pr].y, ARG2_HI));
            }
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const float2 Bp0 = make_float2(B4[r].x, B4[r].y), Bp1 = make_float2(B4[r].z, B4[r].w);
                uint32_t tv[16];
#pragma unroll
                for (int cc = 0; cc < 2; ++cc) {
                    const float2 du2 = f2(dt[r][cc] * uu[r][cc]);
                    const float2 a0 = make_float2(ex2(x[r][cc][0].x), ex2(x[r][cc][0].y));
                    const float2 a1 = make_float2(ex2(x[r][cc][1].x), ex2(x[r][cc][1].y));
                    tv[4 * cc + 0] = __float_as_uint(h[cc][0].x);
                    tv[4 * cc + 1] = __float_as_uint(h[cc][0].y);
                    tv[4 * cc + 2] = __float_as_uint(h[cc][1].x);
                    tv[4 * cc + 3] = __float_as_uint(h[cc][1].y);
                    tv[8 + 4 * cc + 0] = __float_as_uint(a0.x);
                    tv[8 + 4 * cc + 1] = __float_as_uint(a0.y);
                    tv[8 + 4 * cc + 2] = __float_as_uint(a1.x);
                    tv[8 + 4 * cc + 3] = __float_as_uint(a1.y);
                    h[cc][0] = __ffma2_rn(a0, h[cc][0], __fmul2_rn(du2, Bp0));
                    h[cc][1] = __ffma2_rn(a1, h[cc][1], __fmul2_rn(du2, Bp1));
                }
                tmem_st16(tcache + (uint32_t)(i0 + r) * 16u, tv);
            }
        }
        };
        if (a_nonpos && s.dpos[st] != 0)
            recompute(std::false_type{});
        else
            recompute(std::true_type{});
        tmem_wait_st();   // the adjoint pass reads these columns back

        if (pc == 0 && kp > 0) {
            mbar_wait(&s.qfull[st], (qphase >> st) & 1u, p.err);
            qphase ^= 1u << st;
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (dvc[cc]) v = *reinterpret_cast<const float4*>(&s.qin[st][c2 + cc][4 * sg]);
                q[cc][0] = make_float2(v.x, v.y);
                q[cc][1] = make_float2(v.z, v.w);
            }
        }

        // ---- adjoint pass: blocks of 4 steps, last block first. The serial updates run
        //      step by step; the cross-lane sums of a block are batched after it ----
        const int rb = it % RB;
        mbar_wait(&s.redempty[rb], ((unsigned)(it / RB) & 1u) ^ 1u, p.err);
        const int ob = it & 1;
        if constexpr (Cfg::STAGE_OUT) mbar_wait(&s.oempty[ob], ((unsigned)(it / 2) & 1u) ^ 1u, p.err);
        T* dub = static_cast<T*>(p.du);
        T* ddb = static_cast<T*>(p.ddelta);
        __syncwarp();
        float2 ht[2][2];   // state after the step being processed
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
            ht[cc][0] = h[cc][0];
            ht[cc][1] = h[cc][1];
        }
#pragma unroll 1
        for (int i0 = PB_LT - 4; i0 >= 0; i0 -= 4) {
            float dt[4][2], uu[4][2], gy[4][2];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                load2<T>(dt[r], &s.d[st][i0 + r][c2]);
                load2<T>(uu[r], &s.u[st][i0 + r][c2]);
                load2<T>(gy[r], &s.g[st][i0 + r][c2]);
            }
            uint32_t tv[4][16];   // per step: state before the step, then its decay factors
            // only the float32 path's direct output stores diverge inside this loop
            if constexpr (!Cfg::STAGE_OUT) __syncwarp();
#pragma unroll
            for (int r = 0; r < 4; ++r) tmem_ld16(tcache + (uint32_t)(i0 + r) * 16u, tv[r]);
            tmem_wait_ld4(tv);
            float vv[4][8];   // per step: dB partial (states 4sg..4sg+3), then dC partial
            float sv[4][4];   // per step: S1 (channels c2, c2+1), then S2
#pragma unroll
            for (int r = 3; r >= 0; --r) {
                const int i = i0 + r;
                const float4 B4 = *reinterpret_cast<const float4*>(Bf + i * NSTATE + 4 * sg);
                const float4 C4 = *reinterpret_cast<const float4*>(Cf + i * NSTATE + 4 * sg);
                const float2 Bp[2] = {make_float2(B4.x, B4.y), make_float2(B4.z, B4.w)};
                const float2 Cp[2] = {make_float2(C4.x, C4.y), make_float2(C4.z, C4.w)};
                float2 hp[2][2], av[2][2];   // state before step i, decay factors of step i
#pragma unroll
                for (int cc = 0; cc < 2; ++cc)
#pragma unroll
                    for (int pr = 0; pr < 2; ++pr) {
                        hp[cc][pr] = make_float2(__uint_as_float(tv[r][4 * cc + 2 * pr]),
                                                 __uint_as_float(tv[r][4 * cc + 2 * pr + 1]));
                        av[cc][pr] = make_float2(__uint_as_float(tv[r][8 + 4 * cc + 2 * pr]),
                                                 __uint_as_float(tv[r][8 + 4 * cc + 2 * pr + 1]));
                    }
                float2 vB[2], vC[2];
#pragma unroll
                for (int cc = 0; cc < 2; ++cc) {
                    const float2 dt2 = f2(dt[r][cc]);
                    const float2 du2 = f2(dt[r][cc] * uu[r][cc]);
                    const float2 gy2 = f2(gy[r][cc]);
                    float2 s1, s2;
#pragma unroll
                    for (int pr = 0; pr < 2; ++pr) {
                        const float2 g = __ffma2_rn(gy2, Cp[pr], q[cc][pr]);
                        // q_{t-1} = a g, and p = g a h_{t-1} = q_{t-1} h_{t-1} reuses it
                        const float2 qn = __fmul2_rn(av[cc][pr], g);
                        const float2 pp = __fmul2_rn(qn, hp[cc][pr]);
                        s1 = pr == 0 ? __fmul2_rn(A2[cc][pr], pp) : __ffma2_rn(A2[cc][pr], pp, s1);
                        s2 = pr == 0 ? __fmul2_rn(g, Bp[pr]) : __ffma2_rn(g, Bp[pr], s2);
                        dA[cc][pr] = __ffma2_rn(dt2, pp, dA[cc][pr]);
                        vB[pr] = cc == 0 ? __fmul2_rn(g, du2) : __ffma2_rn(g, du2, vB[pr]);
                        vC[pr] = cc == 0 ? __fmul2_rn(gy2, ht[cc][pr]) : __ffma2_rn(gy2, ht[cc][pr], vC[pr]);
                        q[cc][pr] = qn;
                    }
                    sv[r][cc] = s1.x + s1.y;
                    sv[r][2 + cc] = s2.x + s2.y;
                }
                vv[r][0] = vB[0].x; vv[r][1] = vB[0].y; vv[r][2] = vB[1].x; vv[r][3] = vB[1].y;
                vv[r][4] = vC[0].x; vv[r][5] = vC[0].y; vv[r][6] = vC[1].x; vv[r][7] = vC[1].y;
#pragma unroll
                for (int cc = 0; cc < 2; ++cc) {
                    ht[cc][0] = hp[cc][0];
                    ht[cc][1] = hp[cc][1];
                }
            }
            // S1 / S2 over the 4 state groups: reduce-scatter (xor 2, then 1); lane sg
            // ends with the sums of step i0 + sg
            {
                const bool up = (sg & 2) != 0;
#pragma unroll
                for (int r = 0; r < 2; ++r)
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        const float send = up ? sv[r][v] : sv[r + 2][v];
                        const float keep = up ? sv[r + 2][v] : sv[r][v];
                        sv[r][v] = keep + __shfl_xor_sync(FULL, send, 2);
                    }
            }
            {
                const bool up = (sg & 1) != 0;
#pragma unroll
                for (int v = 0; v < 4; ++v) {
                    const float send = up ? sv[0][v] : sv[1][v];
                    const float keep = up ? sv[1][v] : sv[0][v];
                    sv[0][v] = keep + __shfl_xor_sync(FULL, send, 1);
                }
            }
            {
                const int i = i0 + sg;
                float dq[2], uq[2], gq[2];
                load2<T>(dq, &s.d[st][i][c2]);
                load2<T>(uq, &s.u[st][i][c2]);
                load2<T>(gq, &s.g[st][i][c2]);
                const float du0 = fmaf(gq[0], Dd[0], dq[0] * sv[0][2]);
                const float du1 = fmaf(gq[1], Dd[1], dq[1] * sv[0][3]);
                // dD = sum_t dout u: lane sg takes the steps i0 + sg (summed over sg at the unit end)
                dD[0] = fmaf(gq[0], uq[0], dD[0]);
                dD[1] = fmaf(gq[1], uq[1], dD[1]);
                const float dd0 = fmaf(uq[0], sv[0][2], sv[0][0] * LN2);
                const float dd1 = fmaf(uq[1], sv[0][3], sv[0][1] * LN2);
                if constexpr (Cfg::STAGE_OUT) {
                    store2<T>(&s.duo[ob][i][c2], du0, du1);
                    store2<T>(&s.ddo[ob][i][c2], dd0, dd1);
                } else {
                    const int t = t0 + i;
                    if (t < p.L) {
                        const int64_t off = ((int64_t)b * p.L + t) * p.D + dbase;
                        if (dvc[1]) {
                            store2<T>(dub + off, du0, du1);
                            store2<T>(ddb + off, dd0, dd1);
                        } else if (dvc[0]) {
                            dub[off] = from_f<T>(du0);
                            ddb[off] = from_f<T>(dd0);
                        }
                    }
                }
            }
            // dB | dC over the warp's 8 channel pairs: reduce-scatter (xor 16, 8, 4); lane
            // (cg, sg) ends with step i0 + cg / 2, part cg % 2 (dB, dC), states 4sg..4sg+3
            {
                const bool up = (cg & 4) != 0;
#pragma unroll
                for (int r = 0; r < 2; ++r)
#pragma unroll
                    for (int k2 = 0; k2 < 8; ++k2) {
                        const float send = up ? vv[r][k2] : vv[r + 2][k2];
                        const float keep = up ? vv[r + 2][k2] : vv[r][k2];
                        vv[r][k2] = keep + __shfl_xor_sync(FULL, send, 16);
                    }
            }
            {
                const bool up = (cg & 2) != 0;
#pragma unroll
                for (int k2 = 0; k2 < 8; ++k2) {
                    const float send = up ? vv[0][k2] : vv[1][k2];
                    const float keep = up ? vv[1][k2] : vv[0][k2];
                    vv[0][k2] = keep + __shfl_xor_sync(FULL, send, 8);
                }
            }
            {
                const bool up = (cg & 1) != 0;
#pragma unroll
                for (int k2 = 0; k2 < 4; ++k2) {
                    const float send = up ? vv[0][k2] : vv[0][k2 + 4];
                    const float keep = up ? vv[0][k2 + 4] : vv[0][k2];
                    vv[0][k2] = keep + __shfl_xor_sync(FULL, send, 4);
                }
            }
            *reinterpret_cast<float4*>(&s.red[rb][w][i0 + (cg >> 1)][(cg & 1) * NSTATE + 4 * sg]) =
                make_float4(vv[0][0], vv[0][1], vv[0][2], vv[0][3]);
        }
        // inputs of the stage consumed; partials and output tile written
        __syncwarp();
        if (lane == 0) {
            mbar_arrive_b(&s.empty[st]);
            mbar_arrive_b(&s.redfull[rb]);
        }
        if constexpr (Cfg::STAGE_OUT) {
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) mbar_arrive_b(&s.ofull[ob]);
        }

        if (unit_end) {
            const int64_t ub = (int64_t)unit * PB_CPB + c2;
#pragma unroll
            for (int cc = 0; cc < 2; ++cc)
                *reinterpret_cast<float4*>(p.ws_a + (ub + cc) * NSTATE + 4 * sg) =
                    make_float4(dA[cc][0].x, dA[cc][0].y, dA[cc][1].x, dA[cc][1].y);
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {   // the 4 state-group lanes hold every 4th step
                dD[cc] += __shfl_xor_sync(FULL, dD[cc], 1);
                dD[cc] += __shfl_xor_sync(FULL, dD[cc], 2);
            }
            if (sg == 0) *reinterpret_cast<float2*>(p.ws_d + ub) = make_float2(dD[0], dD[1]);
            if (k > 0) {
                if (p.mode == 0) {   // seeded segments find the records already written
                    float* hs = p.hand + ((int64_t)(c * p.K + kp) * PB_CPB + c2) * NSTATE + 4 * sg;
#pragma unroll
                    for (int cc = 0; cc < 2; ++cc)
                        *reinterpret_cast<float4*>(hs + cc * NSTATE) =
                            make_float4(q[cc][0].x, q[cc][0].y, q[cc][1].x, q[cc][1].y);
                    __threadfence();
                    __syncwarp();
                    if (lane == 0) atomicAdd(&p.flags[c * p.K + kp], 1);
                }
            } else if (p.dh_prev != nullptr) {
#pragma unroll
                for (int cc = 0; cc < 2; ++cc)
                    if (dvc[cc]) {
                        const float v4[4] = {q[cc][0].x, q[cc][0].y, q[cc][1].x, q[cc][1].y};
                        store_state4<T>(p.dh_prev, ((int64_t)b * p.D + dbase + cc) * NSTATE + 4 * sg, v4,
                                        p.carry32 != 0);
                    }
            }
        }
    }
    // every compute warp leaves the loop on the same (terminating) stage; then warp 0 frees
    // the TMEM columns (warp-collective: reconverge first)
    __syncwarp();
    tmem_fence_before_sync();
    asm volatile("bar.sync 1, %0;" ::"n"(PB_NCT) : "memory");
    if (w == 0) {
        tmem_fence_after_sync();
        tmem_dealloc(s.tmem_base, PB_TMEM_COLS);
    }
}

// Fixed-order sums of the persistent backward's partials into dA, dD (over batch rows and
// segments) and dB, dC (over channel blocks).
template <typename T>
__global__ void ss_bwd_persistent_final_kernel(const __grid_constant__ PBwdArgs p, void* dA_,
                                               void* dB_, void* dC_, void* dD_) {
    const int64_t Lp = (int64_t)p.nck * CK;
    const int64_t n_bc = (int64_t)p.B * p.L * p.G * 2 * NSTATE;
    const int64_t n_a = (int64_t)p.D * NSTATE;
    const int bpg = p.G > 1 ? p.cpg / PB_CPB : p.nblk;   // blocks per B / C group
    const int64_t total = n_bc + n_a + p.D;
    T* dA = static_cast<T*>(dA_);
    T* dB = static_cast<T*>(dB_);
    T* dC = static_cast<T*>(dC_);
    T* dD = static_cast<T*>(dD_);
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        if (idx < n_bc) {
            // (b, t, g, v): the sum over the 128-channel blocks of group g, in block order
            const int64_t v = idx % (2 * NSTATE);
            const int64_t btg = idx / (2 * NSTATE);
            const int g = (int)(btg % p.G);
            const int64_t bt = btg / p.G;
            const int64_t b = bt / p.L, t = bt % p.L;
            float s = 0.f;
            for (int blk = g * bpg; blk < (g + 1) * bpg; ++blk)
                s += p.ws_bc[(((int64_t)b * Lp + t) * p.nblk + blk) * (2 * NSTATE) + v];
            if (v < NSTATE) dB[btg * NSTATE + v] = from_f<T>(s);
            else dC[btg * NSTATE + v - NSTATE] = from_f<T>(s);
        } else {
            const bool isA = idx < n_bc + n_a;
            const int64_t i = isA ? idx - n_bc : idx - n_bc - n_a;
            const int64_t d = isA ? i / NSTATE : i;
            const int n = isA ? (int)(i % NSTATE) : 0;
            const int blk = (int)(d / PB_CPB), ch = (int)(d % PB_CPB);
            float s = 0.f;
            for (int kp = 0; kp < p.K; ++kp)
                for (int b = 0; b < p.B; ++b) {
                    const int64_t unit = (int64_t)kp * p.nchains + b * p.nblk + blk;
                    s += isA ? p.ws_a[(unit * PB_CPB + ch) * NSTATE + n] : p.ws_d[unit * PB_CPB + ch];
                }
            if (isA) dA[i] = from_f<T>(s);
            else dD[i] = from_f<T>(s);
        }
    }
}

// ------------------------------------------------------------ few-chain split passes
// Pass 1: for segment k >= 1 of chain c (unit kp = K-1-k, walked last step first), the
// adjoint state at the segment's start when q = 0 at its end (dh_last for the last segment):
//   q <- a_t (dout_t C_t + q),  a_t = 2^(delta_t A log2 e)   (the reference's adjoint without
// the gradient terms, mamba_windows_cuda/mamba_cuda.py:703-742), and the segment's delta sum.
// Thread = (channel, half): 8 of the channel's 16 states as packed float2 pairs; the CTA
// stages 32-step tiles of delta / dout (32 x 128, 16-byte vectors: rows of D * elem are
// 16-byte multiples on this path) and C (32 x 16, float32) in shared memory, each thread
// loading its share of the next tile into registers while the current one is computed.
constexpr int AJ_LT = 32;

template <typename T>
__global__ void __launch_bounds__(256) ss_bwd_adjoint_kernel(
    const T* __restrict__ delta, const T* __restrict__ dout, const T* __restrict__ Cm, const T* __restrict__ A,
    const void* __restrict__ dh_last, float* __restrict__ hand, float* __restrict__ segsum, int L, int D,
    int nblk, int nchains, int K, int seg_tiles, int G, int cpg, int carry32) {
    constexpr int VE = 16 / (int)sizeof(T);   // elements per 16-byte vector
    constexpr int VPR = PB_CPB / VE;          // vectors per 128-channel row
    __shared__ __align__(16) T sd[AJ_LT][PB_CPB];
    __shared__ __align__(16) T sgy[AJ_LT][PB_CPB];
    __shared__ __align__(16) float sC[AJ_LT][NSTATE];
    const int unit = blockIdx.x;   // kp * nchains + c
    const int c = unit % nchains, kp = unit / nchains, k = K - 1 - kp;
    const int b = c / nblk, blk = c % nblk;
    const int grp = blk * PB_CPB / cpg;   // the block's C group
    const int tstart = k * seg_tiles * PB_LT;
    const int tend = min(tstart + seg_tiles * PB_LT, L);
    const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
    const int ch = w * 16 + (lane >> 1), n0 = (lane & 1) * 8;
    const int64_t d = (int64_t)blk * PB_CPB + ch;
    const bool dv = d < D;
    float2 A2[4], q[4];
    bool a_nonpos = true;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        float av[2], qv[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int n = n0 + 2 * j + e;
            av[e] = dv ? to_f(A[d * NSTATE + n]) * LOG2E : 0.f;
            const int64_t off = ((int64_t)b * D + d) * NSTATE + n;
            qv[e] = (kp == 0 && dh_last != nullptr && dv)
                        ? (carry32 ? static_cast<const float*>(dh_last)[off] : to_f(static_cast<const T*>(dh_last)[off]))
                        : 0.f;
            a_nonpos = a_nonpos && av[e] <= 0.f;
        }
        A2[j] = make_float2(av[0], av[1]);
        q[j] = make_float2(qv[0], qv[1]);
    }
    float sumd = 0.f;
    const int ntl = (tend - tstart + AJ_LT - 1) / AJ_LT;
    // This thread's share of a tile, loaded into registers one tile ahead (the next tile's
    // loads are in flight while the current one is computed).
    constexpr int NV = AJ_LT * VPR / 256;       // 16-byte vectors per tensor and thread
    constexpr int NCE = AJ_LT * NSTATE / 256;   // C elements per thread
    static_assert(AJ_LT * VPR % 256 == 0 && AJ_LT * NSTATE % 256 == 0, "whole tiles per CTA");
    uint4 ra[NV], rg[NV];
    float rc[NCE];
    bool rneg = false;   // a delta of the prefetched share has its sign bit set
    auto fetch = [&](int ti) {
        const int t0 = tstart + ti * AJ_LT;
        const int nr = min(AJ_LT, tend - t0);
        rneg = false;
#pragma unroll
        for (int v = 0; v < NV; ++v) {
            const int idx = tid + v * 256, r = idx / VPR, col = idx % VPR;
            const int64_t dd = (int64_t)blk * PB_CPB + col * VE;
            ra[v] = make_uint4(0u, 0u, 0u, 0u);
            rg[v] = ra[v];
            if (r < nr && dd < D) {
                const int64_t off = ((int64_t)b * L + t0 + r) * D + dd;
                ra[v] = *reinterpret_cast<const uint4*>(delta + off);
                rg[v] = *reinterpret_cast<const uint4*>(dout + off);
            }
            constexpr uint32_t SIGN = sizeof(T) == 2 ? 0x80008000u : 0x80000000u;
            rneg = rneg || (((ra[v].x | ra[v].y | ra[v].z | ra[v].w) & SIGN) != 0u);
        }
#pragma unroll
        for (int e = 0; e < NCE; ++e) {
            const int idx = tid + e * 256, r = idx / NSTATE, n = idx % NSTATE;
            rc[e] = r < nr ? to_f(Cm[(((int64_t)b * L + t0 + r) * G + grp) * NSTATE + n]) : 0.f;
        }
    };
    if (ntl > 0) fetch(ntl - 1);
    for (int ti = ntl - 1; ti >= 0; --ti) {
        const int t0 = tstart + ti * AJ_LT;
        const int nr = min(AJ_LT, tend - t0);
        __syncthreads();   // the previous tile is no longer read
#pragma unroll
        for (int v = 0; v < NV; ++v) {
            const int idx = tid + v * 256, r = idx / VPR, col = idx % VPR;
            *reinterpret_cast<uint4*>(&sd[r][col * VE]) = ra[v];
            *reinterpret_cast<uint4*>(&sgy[r][col * VE]) = rg[v];
        }
#pragma unroll
        for (int e = 0; e < NCE; ++e) {
            const int idx = tid + e * 256;
            sC[idx / NSTATE][idx % NSTATE] = rc[e];
        }
        // the tile is in shared memory; the exponent clamp is the identity for the whole tile
        // when no delta of it is negative and A <= 0 for every channel of the CTA
        const bool noclamp = __syncthreads_and(!rneg && a_nonpos) != 0;
        if (ti > 0) fetch(ti - 1);
        auto steps = [&](auto clamp_tag) {
            constexpr bool CLAMP = decltype(clamp_tag)::value;
#pragma unroll 4
            for (int r = nr - 1; r >= 0; --r) {
                const float dt = to_f(sd[r][ch]), gy = to_f(sgy[r][ch]);
                sumd += dt;
                const float2 dt2 = make_float2(dt, dt), gy2 = make_float2(gy, gy);
                const float4* Cq = reinterpret_cast<const float4*>(&sC[r][n0]);
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const float4 c4 = Cq[h];
                    const float2 cp[2] = {make_float2(c4.x, c4.y), make_float2(c4.z, c4.w)};
#pragma unroll
                    for (int j = 0; j < 2; ++j) {
                        const int jj = 2 * h + j;
                        float2 x = __fmul2_rn(dt2, A2[jj]);
                        if constexpr (CLAMP) x = make_float2(fminf(x.x, ARG2_HI), fminf(x.y, ARG2_HI));
                        const float2 a = make_float2(ex2(x.x), ex2(x.y));
                        q[jj] = __fmul2_rn(a, __ffma2_rn(gy2, cp[j], q[jj]));
                    }
                }
            }
        };
        if (noclamp) steps(std::false_type{});
        else steps(std::true_type{});
    }
    float qs[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        qs[2 * j] = q[j].x;
        qs[2 * j + 1] = q[j].y;
    }
    float* rec = hand + ((int64_t)(c * K + kp) * PB_CPB + ch) * NSTATE + n0;
#pragma unroll
    for (int j = 0; j < 8; ++j) rec[j] = qs[j];
    if ((lane & 1) == 0) segsum[(int64_t)(c * K + kp) * PB_CPB + ch] = sumd;
}

// Fold of the adjoint records in reverse time: record kp (segment K-1-kp) holds q at the
// segment's start from q = 0 at its end (the last segment from dh_last, so record 0 is
// exact); afterwards record kp holds the true q at that point:
//   Q_kp = 2^(A log2(e) * sumd_kp) Q_{kp-1} + R_kp   (a segment's decay is exp(A * sum delta))
template <typename T>
__global__ void ss_bwd_fold_kernel(float* __restrict__ hand, const float* __restrict__ segsum,
                                   const T* __restrict__ A, int nblk, int nchains, int K, int D) {
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;   // (c, ch, n), n fastest
    if (tid >= (int64_t)nchains * PB_CPB * NSTATE) return;
    const int n = (int)(tid % NSTATE);
    const int ch = (int)((tid / NSTATE) % PB_CPB);
    const int c = (int)(tid / (NSTATE * PB_CPB));
    const int64_t d = (int64_t)(c % nblk) * PB_CPB + ch;
    const float a2 = d < D ? to_f(A[d * NSTATE + n]) * LOG2E : 0.f;
    float* r = hand + ((int64_t)c * K * PB_CPB + ch) * NSTATE + n;
    const float* sm = segsum + (int64_t)c * K * PB_CPB + ch;
    float Q = r[0];
    for (int kp = 1; kp < K - 1; ++kp) {
        Q = fmaf(ex2(fminf(a2 * sm[(int64_t)kp * PB_CPB], ARG2_HI)), Q, r[(int64_t)kp * PB_CPB * NSTATE]);
        r[(int64_t)kp * PB_CPB * NSTATE] = Q;
    }
}

PersistPlan plan_persistent_bwd_split(int64_t B, int64_t L, int64_t D, int num_sms) {
    PersistPlan pl{};
    pl.nblk = (int)((D + PB_CPB - 1) / PB_CPB);
    pl.nchains = (int)(B * pl.nblk);
    pl.ntiles = (int)((L + PB_LT - 1) / PB_LT);
    pl.ok = false;
    // below ~512 steps one generic pass is as fast as three short launches
    if (pl.nchains <= 0 || pl.nchains >= num_sms || (int64_t)pl.ntiles * PB_LT < 512) return pl;
    const int K = pick_split_segments(pl.nchains, pl.ntiles, num_sms, 2);
    if (K < 2) return pl;
    pl.K = K;
    pl.seg_tiles = (pl.ntiles + K - 1) / K;
    pl.grid = (int)std::min<int64_t>(num_sms, (int64_t)pl.nchains * K);
    pl.ok = true;
    return pl;
}

PersistPlan plan_persistent_bwd(int64_t B, int64_t L, int64_t D, int num_sms) {
    PersistPlan pl{};
    pl.nblk = (int)((D + PB_CPB - 1) / PB_CPB);
    pl.nchains = (int)(B * pl.nblk);
    pl.ntiles = (int)((L + PB_LT - 1) / PB_LT);
    pl.ok = pl.nchains >= num_sms;
    int best_k = 1;
    double best = -1.0;
    for (int K = 1; K <= pl.ntiles; ++K) {
        const int seg = (pl.ntiles + K - 1) / K;
        if ((pl.ntiles + seg - 1) / seg != K) continue;
        if (K > 1 && seg < MWC_BWD_MIN_SEG_TILES) break;
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

// Workspace: [counter, err, flags | hand | ws_a | ws_d | ws_bc], 256-byte aligned parts.
BwdPersistWs bwd_persistent_ws(const PersistPlan& pl, int64_t B, int64_t L) {
    BwdPersistWs w{};
    const int64_t units = (int64_t)pl.nchains * pl.K;
    auto up = [](int64_t x) { return (x + 255) / 256 * 256; };
    w.off_hand = up(16 + units * 4);
    w.off_a = w.off_hand + up(units * PB_CPB * NSTATE * 4);
    w.off_d = w.off_a + up(units * PB_CPB * NSTATE * 4);
    w.off_bc = w.off_d + up(units * PB_CPB * 4);
    const int64_t Lp = (L + CK - 1) / CK * CK;
    w.off_sum = w.off_bc + up((int64_t)pl.nblk * B * Lp * 2 * NSTATE * 4);
    w.total = w.off_sum + up(units * PB_CPB * 4);   // per-segment delta sums (split passes)
    return w;
}

static_assert(sizeof(PBwdSmem<float>) <= 227 * 1024 && sizeof(PBwdSmem<__half>) <= 227 * 1024 &&
                  sizeof(PBwdSmem<__nv_bfloat16>) <= 227 * 1024,
              "backward shared memory exceeds the 227 KB a CTA may use");

template <typename T>
static cudaError_t launch_pb(const PBwdArgs& a, int grid, void* dA, void* dB, void* dC, void* dD,
                             cudaStream_t s) {
    // more than half of the SM's shared memory: one CTA per SM, so the CTA's 512-column TMEM
    // allocation never waits for another CTA of this kernel
    const size_t smem = std::max(sizeof(PBwdSmem<T>), (size_t)(120 * 1024));
    cudaError_t e = ensure_smem_attr<ss_bwd_persistent_kernel<T>>((int)smem);
    if (e != cudaSuccess) return e;
    ss_bwd_persistent_kernel<T><<<grid, PB_NT, smem, s>>>(a);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const int64_t total = (int64_t)a.B * a.L * a.G * 2 * NSTATE + (int64_t)a.D * NSTATE + a.D;
    int64_t blocks = std::min<int64_t>((total + 255) / 256, 148 * 8);
    ss_bwd_persistent_final_kernel<T><<<(unsigned)std::max<int64_t>(blocks, 1), 256, 0, s>>>(a, dA, dB, dC, dD);
    return cudaGetLastError();
}

cudaError_t launch_bwd_persistent(PBwdArgs& a, const PersistPlan& pl, int dtype, void* ws,
                                  void* dA, void* dB, void* dC, void* dD, cudaStream_t s) {
    const BwdPersistWs w = bwd_persistent_ws(pl, a.B, a.L);
    char* base = static_cast<char*>(ws);
    a.counter = reinterpret_cast<int*>(base);
    a.err = reinterpret_cast<int*>(base + 4);
    a.flags = reinterpret_cast<int*>(base + 16);
    a.hand = reinterpret_cast<float*>(base + w.off_hand);
    a.ws_a = reinterpret_cast<float*>(base + w.off_a);
    a.ws_d = reinterpret_cast<float*>(base + w.off_d);
    a.ws_bc = reinterpret_cast<float*>(base + w.off_bc);
    a.nblk = pl.nblk;
    a.nchains = pl.nchains;
    a.K = pl.K;
    a.seg_tiles = pl.seg_tiles;
    a.ntiles = pl.ntiles;
    cudaError_t e = cudaMemsetAsync(ws, 0, (size_t)w.off_hand, s);
    if (e != cudaSuccess) return e;
    if (dtype == 2) return launch_pb<__nv_bfloat16>(a, pl.grid, dA, dB, dC, dD, s);
    return dtype == 1 ? launch_pb<__half>(a, pl.grid, dA, dB, dC, dD, s)
                      : launch_pb<float>(a, pl.grid, dA, dB, dC, dD, s);
}

// Few chains: the adjoint-only pass over segments K-1..1, the fold, then the ordinary
// backward with every segment seeded from its record (mode 2).
template <typename T>
static cudaError_t bwd_split_passes(PBwdArgs& a, const PersistPlan& pl, float* segsum, const void* delta,
                                    const void* dout, const void* Cm, void* dA, void* dB, void* dC, void* dD,
                                    cudaStream_t s) {
    const T* At = static_cast<const T*>(a.A);
    ss_bwd_adjoint_kernel<T><<<(unsigned)(pl.nchains * (pl.K - 1)), 256, 0, s>>>(
        static_cast<const T*>(delta), static_cast<const T*>(dout), static_cast<const T*>(Cm), At,
        a.dh_last, a.hand, segsum, a.L, a.D, pl.nblk, pl.nchains, pl.K, pl.seg_tiles, a.G, a.cpg,
        a.carry32);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const int64_t nthr = (int64_t)pl.nchains * PB_CPB * NSTATE;
    ss_bwd_fold_kernel<T><<<(unsigned)((nthr + 255) / 256), 256, 0, s>>>(a.hand, segsum, At, pl.nblk, pl.nchains,
                                                                       pl.K, a.D);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    return launch_pb<T>(a, pl.grid, dA, dB, dC, dD, s);
}

cudaError_t launch_bwd_persistent_split(PBwdArgs& a, const PersistPlan& pl, int dtype, void* ws,
                                        const void* delta, const void* dout, const void* Cm,
                                        void* dA, void* dB, void* dC, void* dD, cudaStream_t s) {
    const BwdPersistWs w = bwd_persistent_ws(pl, a.B, a.L);
    char* base = static_cast<char*>(ws);
    a.counter = reinterpret_cast<int*>(base);
    a.err = reinterpret_cast<int*>(base + 4);
    a.flags = reinterpret_cast<int*>(base + 16);
    a.hand = reinterpret_cast<float*>(base + w.off_hand);
    a.ws_a = reinterpret_cast<float*>(base + w.off_a);
    a.ws_d = reinterpret_cast<float*>(base + w.off_d);
    a.ws_bc = reinterpret_cast<float*>(base + w.off_bc);
    float* segsum = reinterpret_cast<float*>(base + w.off_sum);
    a.nblk = pl.nblk;
    a.nchains = pl.nchains;
    a.K = pl.K;
    a.seg_tiles = pl.seg_tiles;
    a.ntiles = pl.ntiles;
    a.mode = 2;
    cudaError_t e = cudaMemsetAsync(ws, 0, (size_t)w.off_hand, s);
    if (e != cudaSuccess) return e;
    if (dtype == 2) return bwd_split_passes<__nv_bfloat16>(a, pl, segsum, delta, dout, Cm, dA, dB, dC, dD, s);
    if (dtype == 1) return bwd_split_passes<__half>(a, pl, segsum, delta, dout, Cm, dA, dB, dC, dD, s);
    return bwd_split_passes<float>(a, pl, segsum, delta, dout, Cm, dA, dB, dC, dD, s);
}

}  // namespace mwc
