// Persistent, warp-specialized, TMA-pipelined forward selective scan for sm_100a.
//
// Work decomposition: a "chain" is one batch row x 128 channels over all of L, cut into
// 32-step tiles. With at least as many chains as SMs (the chained path, mode 0), one
// persistent CTA per SM takes an equal run of the chains' concatenated tiles (config 3:
// 160 chains x 64 tiles on 148 SMs, 69-70 tiles per CTA). A chain cut between two runs is
// handed over once: the earlier run scans that chain's head first and publishes its end
// state (8 per-warp release increments of a flag); the later run scans the chain's tail
// last, so the record is ready or nearly ready when it is needed (each wait is bounded).
// A dynamic queue of K time segments per chain instead leaves no slack when the chains
// barely outnumber the SMs: most units start one wave after the unit they depend on.
// With fewer chains than SMs the split passes (modes 1 / 2) take K independent segments
// per chain from an atomic queue.
//
// CTA = 10 warps, no CTA-wide barrier after set-up; mbarriers connect the roles:
//   * warps 0-7 (compute): thread = (channel, half): 8 of the channel's 16 states in
//     registers as 4 float2 pairs (packed FFMA2), the two halves' <C, h> meet through one
//     shuffle; ex2 with log2(e) folded into A; y to a staging tile, float32 checkpoints
//     every 16 steps straight to global memory;
//   * warp 8 (producer): the CTA's units, hand-off waits, TMA loads of u / delta (32 x 128),
//     B / C (32 x 16) and the segment's incoming state (1-D bulk copy) into a ring of
//     stages (full / empty mbarriers);
//   * warp 9 (helper): float32 copies of B / C for fp16 inputs, and the TMA stores of y
//     from the double-buffered staging tile.
#include "mwc_device.cuh"
#include "mwc_internal.h"
#include "mwc_tma.cuh"

#include <cudaTypedefs.h>

#include <algorithm>
#include <type_traits>

namespace mwc {

constexpr int PF_LT = 32;
constexpr int PF_CPB = 128;
#ifndef MWC_FWD_SPT
#define MWC_FWD_SPT 8   // states per compute thread: 8 (8 compute warps; 4 with 16 warps measured slower)
#endif
constexpr int PF_SPT = MWC_FWD_SPT;
constexpr int PF_NP = PF_SPT / 2;            // float2 state pairs per thread
constexpr int PF_LPC = NSTATE / PF_SPT;      // lanes per channel
constexpr int PF_NCW = PF_CPB * PF_LPC / 32; // compute warps
constexpr int PF_NT = (PF_NCW + 2) * 32;     // + producer warp + helper warp
constexpr int PF_HAND = PF_CPB * (NSTATE + 1);  // floats of one segment hand-off record
static_assert(PF_LT % CK == 0, "a forward tile holds whole checkpoint chunks");
#ifndef MWC_FWD_SPLIT_MIN_SEG_TILES
#define MWC_FWD_SPLIT_MIN_SEG_TILES 2   // shortest independent segment of the few-chain split
#endif

template <typename T>
struct PfCfg {
    static constexpr int ST = sizeof(T) == 2 ? 4 : 3;   // pipeline depth (stages)
};

template <typename T>
struct __align__(128) PFwdSmem {
    static constexpr int ST = PfCfg<T>::ST;
    T u[ST][PF_LT][PF_CPB];
    T d[ST][PF_LT][PF_CPB];
    T Bt[ST][PF_LT][NSTATE];
    T Ct[ST][PF_LT][NSTATE];
    T y[2][PF_LT][PF_CPB];                                       // y staging for TMA stores
    float hin[ST][PF_HAND];                                      // incoming segment state
    T At[ST][PF_CPB][NSTATE];                                    // unit parameters: A rows,
    T Ht[ST][PF_CPB][NSTATE];                                    // h_prev rows,
    T Dt[ST][PF_CPB];                                            // D
    float Bf[sizeof(T) == 2 ? ST : 1][PF_LT][NSTATE];            // float32 B / C (fp16 only)
    float Cf[sizeof(T) == 2 ? ST : 1][PF_LT][NSTATE];
    uint64_t full[ST], conv[ST], empty[ST], yfull[2], yempty[2];
    // the stage's unit: chain (-1: no more units), tile within the unit, the unit's first
    // tile in the chain and its tile count, where its incoming state comes from (RIN_*, or a
    // record index) and where its end state goes (ROUT_*, or a record index)
    int unit[ST];
    int tile[ST];
    int first[ST], ntl[ST], rin[ST], rout[ST];
    int dpos[ST];   // helper: 1 when no delta of the stage's tile has its sign bit set
};

constexpr int RIN_START = -2;   // the chain's start: h_prev (or zero)
constexpr int RIN_ZERO = -1;    // zero (state-only segments after the first)
constexpr int ROUT_END = -1;    // the chain's end: h_last / decay
constexpr int ROUT_NONE = -2;   // nothing (seeded segments before the last)

// One block of 8 steps for the lane's 8 states (4 float2 pairs). CLAMP applies the
// safe_exp upper clamp per state; the caller takes the unclamped variant only when every
// exponent of the block is provably <= 0 (A <= 0 and delta >= 0), where the clamp is the
// identity.
template <bool CLAMP>
__device__ __forceinline__ void fwd_block8(float2 (&h2)[PF_NP], const float2 (&A2v)[PF_NP],
                                           const float (&dtv)[8], const float (&uv)[8],
                                           const float* Bf, const float* Cf, int n0,
                                           float (&yv)[8]) {
    constexpr int NQ = PF_NP / 2;   // float4 groups of the lane's states
#pragma unroll
    for (int r = 0; r < 8; ++r) {
        const float2 dt2 = make_float2(dtv[r], dtv[r]);
        const float du = dtv[r] * uv[r];
        const float2 du2 = make_float2(du, du);
        float2 a2[PF_NP];
#pragma unroll
        for (int j = 0; j < PF_NP; ++j) {
            const float2 x = __fmul2_rn(dt2, A2v[j]);
            a2[j] = CLAMP ? make_float2(ex2(fminf(x.x, ARG2_HI)), ex2(fminf(x.y, ARG2_HI)))
                          : make_float2(ex2(x.x), ex2(x.y));
        }
        const float4* Bq = reinterpret_cast<const float4*>(Bf + r * NSTATE + n0);
        const float4* Cq = reinterpret_cast<const float4*>(Cf + r * NSTATE + n0);
        float2 yq[NQ];
#pragma unroll
        for (int q = 0; q < NQ; ++q) {
            const float4 bq = Bq[q];
            const float4 cq = Cq[q];
            h2[2 * q] = __ffma2_rn(a2[2 * q], h2[2 * q], __fmul2_rn(du2, make_float2(bq.x, bq.y)));
            h2[2 * q + 1] =
                __ffma2_rn(a2[2 * q + 1], h2[2 * q + 1], __fmul2_rn(du2, make_float2(bq.z, bq.w)));
            yq[q] = __fmul2_rn(make_float2(cq.x, cq.y), h2[2 * q]);
            yq[q] = __ffma2_rn(make_float2(cq.z, cq.w), h2[2 * q + 1], yq[q]);
        }
        float2 y2 = yq[0];
#pragma unroll
        for (int q = 1; q < NQ; ++q) y2 = __fadd2_rn(y2, yq[q]);
        yv[r] = y2.x + y2.y;
    }
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void bulk_load_1d(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// DECAY: the launch asks for the segment decay, so each lane also sums its channel's delta
// (and passes the sum between segments); without it that work is compiled out.
template <typename T, bool DECAY>
__global__ void __launch_bounds__(PF_NT, 1) ss_fwd_persistent_kernel(const __grid_constant__ PFwdArgs p) {
    // Direct cast (no integer round trip): accesses stay in the shared address space.
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    PFwdSmem<T>& s = *reinterpret_cast<PFwdSmem<T>*>(smem_raw);
    constexpr int ST = PfCfg<T>::ST;
    constexpr bool HALF = sizeof(T) == 2;
    if ((smem_u32(smem_raw) & 127u) != 0u) {  // TMA destinations need 128-byte alignment
        if (threadIdx.x == 0) atomicCAS(p.err, 0, ERR_SMEM_ALIGN);
        return;
    }
    const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;

    if (tid == 0) {
        for (int i = 0; i < ST; ++i) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.conv[i], 1);
            mbar_init(&s.empty[i], PF_NCW);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s.yfull[i], PF_NCW);
            mbar_init(&s.yempty[i], 1);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (w == PF_NCW) {
        // ============================== producer ==============================
        if (lane != 0) return;
        prefetch_tmap(&p.tm_u);
        prefetch_tmap(&p.tm_d);
        prefetch_tmap(&p.tm_B);
        prefetch_tmap(&p.tm_C);
        const unsigned tile_bytes =
            (unsigned)((2 * PF_LT * PF_CPB + (p.has_out ? 2 : 1) * PF_LT * NSTATE) * sizeof(T));
        // the unit being issued: chain pc, tiles pfirst .. pfirst + pntl - 1 of it, the source
        // of its incoming state (prin) and the destination of its end state (prout)
        int pc = -1, ptile = 0, pfirst = 0, pntl = 0, prin = RIN_START, prout = ROUT_END;
        // Chained (mode 0): static runs. The chains' tiles, concatenated, are cut into one
        // equal run per CTA, [rs, re); a run is at least one chain long, so a chain is cut at
        // most once, into a head (ending a run) and a tail (starting the next). A run issues
        // the head it ends with first (its record is what the next run's tail waits for), then
        // its whole chains, then the tail it starts with: every tail then waits for a head
        // that the previous run finished first. Run indices come from the counter in the
        // order the CTAs start, so the run a tail waits for belongs to a CTA already running.
        int64_t rs = 0, re = 0;
        int nxt = 0;   // units of the run issued so far
        if (p.mode == 0) {
            const int64_t all = (int64_t)p.nchains * p.ntiles;
            const int64_t r = atomicAdd(p.counter, 1);
            rs = all * r / gridDim.x;
            re = all * (r + 1) / gridDim.x;
        }
        const int total = p.nchains * (p.mode == 1 ? p.K - 1 : p.K);   // state-only: no last segment
        auto next_unit = [&]() -> bool {
            if (p.mode == 0) {
                if (rs >= re) return false;
                const int c_lo = (int)(rs / p.ntiles), c_hi = (int)((re - 1) / p.ntiles);
                const int tail = (int)(rs % p.ntiles), head = (int)(re % p.ntiles);
                const int f_lo = c_lo + (tail != 0 ? 1 : 0), f_hi = c_hi - (head != 0 ? 1 : 0);
                int j = nxt++;
                if (head != 0) {
                    if (j == 0) {
                        pc = c_hi; pfirst = 0; pntl = head; prin = RIN_START; prout = c_hi;
                        return true;
                    }
                    --j;
                }
                if (j <= f_hi - f_lo) {
                    pc = f_lo + j; pfirst = 0; pntl = p.ntiles; prin = RIN_START; prout = ROUT_END;
                    return true;
                }
                if (tail != 0 && j == f_hi - f_lo + 1) {
                    pc = c_lo; pfirst = tail; pntl = p.ntiles - tail; prin = c_lo; prout = ROUT_END;
                    return true;
                }
                return false;
            }
            // split passes (modes 1 / 2): K independent segments per chain from the queue
            const int pu = atomicAdd(p.counter, 1);
            if (pu >= total) return false;
            const int k = pu / p.nchains;
            pc = pu % p.nchains;
            pfirst = k * p.seg_tiles;
            pntl = min(p.seg_tiles, p.ntiles - pfirst);
            prin = k == 0 ? RIN_START : p.mode == 1 ? RIN_ZERO : pc * p.K + k - 1;
            prout = k == p.K - 1 ? ROUT_END : p.mode == 1 ? pc * p.K + k : ROUT_NONE;
            return true;
        };
        for (int it = 0;; ++it) {
            const int st = it % ST;
            mbar_wait(&s.empty[st], ((unsigned)(it / ST) & 1u) ^ 1u, p.err);
            if (pc < 0 || ptile == pntl) {
                if (!next_unit()) {
                    s.unit[st] = -1;
                    mbar_arrive(&s.full[st]);
                    return;
                }
                ptile = 0;
            }
            const int b = pc / p.nblk, blk = pc % p.nblk;
            const int t0 = (pfirst + ptile) * PF_LT;
            s.unit[st] = pc;
            s.tile[st] = ptile;
            s.first[st] = pfirst;
            s.ntl[st] = pntl;
            s.rin[st] = prin;
            s.rout[st] = prout;
            unsigned bytes = tile_bytes;
            const bool need_hand = ptile == 0 && prin >= 0;
            const bool need_hprev = ptile == 0 && prin == RIN_START && p.h_prev != nullptr;
            const int nch = min(PF_CPB, p.D - blk * PF_CPB);
            const unsigned rows_bytes = (unsigned)(nch * NSTATE * sizeof(T));
            if (ptile == 0) bytes += rows_bytes + (unsigned)(nch * sizeof(T));
            if (need_hprev) bytes += rows_bytes;
            if (need_hand) {
                if (p.mode == 0) flag_wait(&p.flags[prin], PF_NCW, p.err);
                // the record was written with generic-proxy stores (made visible by the
                // acquire above); the bulk copy below reads it through the async proxy
                fence_proxy_async_global();
                bytes += PF_HAND * 4;
            }
            mbar_expect_tx(&s.full[st], bytes);
            if (ptile == 0) {
                bulk_load_1d(&s.At[st][0][0], static_cast<const T*>(p.A) + (int64_t)blk * PF_CPB * NSTATE,
                             rows_bytes, &s.full[st]);
                bulk_load_1d(&s.Dt[st][0], static_cast<const T*>(p.Dv) + (int64_t)blk * PF_CPB,
                             (unsigned)(nch * sizeof(T)), &s.full[st]);
            }
            if (need_hprev)
                bulk_load_1d(&s.Ht[st][0][0],
                             static_cast<const T*>(p.h_prev) + ((int64_t)b * p.D + (int64_t)blk * PF_CPB) * NSTATE,
                             rows_bytes, &s.full[st]);
            tma_load_3d(&s.u[st][0][0], &p.tm_u, &s.full[st], blk * PF_CPB, t0, b);
            tma_load_3d(&s.d[st][0][0], &p.tm_d, &s.full[st], blk * PF_CPB, t0, b);
            // the block's B / C group (a 128-channel block lies inside one group)
            const int gx = (blk * PF_CPB / p.cpg) * NSTATE;
            tma_load_3d(&s.Bt[st][0][0], &p.tm_B, &s.full[st], gx, t0, b);
            if (p.has_out) tma_load_3d(&s.Ct[st][0][0], &p.tm_C, &s.full[st], gx, t0, b);
            if (need_hand)
                bulk_load_1d(&s.hin[st][0], p.hand + (int64_t)prin * PF_HAND, PF_HAND * 4, &s.full[st]);
            ++ptile;
        }
    }

    if (w == PF_NCW + 1) {
        // ============== helper: float32 B / C, TMA stores of y ==============
        prefetch_tmap(&p.tm_y);
        int pb = 0, pblk = 0, pt0 = 0;
        for (int it = 0;; ++it) {
            const int st = it % ST;
            mbar_wait(&s.full[st], (unsigned)(it / ST) & 1u, p.err);
            const int unit = s.unit[st];
            int b = 0, blk = 0, t0 = 0;
            if (unit >= 0) {
                b = unit / p.nblk;
                blk = unit % p.nblk;
                t0 = (s.first[st] + s.tile[st]) * PF_LT;
                if constexpr (HALF) {
                    for (int idx = lane; idx < PF_LT * NSTATE; idx += 32) {
                        (&s.Bf[st][0][0])[idx] = to_f((&s.Bt[st][0][0])[idx]);
                        if (p.has_out) (&s.Cf[st][0][0])[idx] = to_f((&s.Ct[st][0][0])[idx]);
                    }
                }
                // safe_exp's clamp is the identity for the whole tile when no delta is
                // negative (given A <= 0): OR of the raw sign bits of the delta tile
                const uint4* dw = reinterpret_cast<const uint4*>(&s.d[st][0][0]);
                constexpr int NW4 = PF_LT * PF_CPB * (int)sizeof(T) / 16;
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
            if (lane == 0) mbar_arrive(&s.conv[st]);
            if (it > 0 && p.has_out) {
                const int yb = (it - 1) & 1;
                mbar_wait(&s.yfull[yb], (unsigned)((it - 1) / 2) & 1u, p.err);
                if (lane == 0) {
                    tma_store_3d(&p.tm_y, &s.y[yb][0][0], pblk * PF_CPB, pt0, pb);
                    bulk_commit();
                    bulk_wait_read0();
                    mbar_arrive(&s.yempty[yb]);
                }
                __syncwarp();
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
    const int half = lane % PF_LPC;   // the lane's share of the channel's states
    const int ch = w * (32 / PF_LPC) + lane / PF_LPC;
    const int n0 = half * PF_SPT;
    float2 A2v[PF_NP], h2[PF_NP];
    float sumd = 0.f, Dd = 0.f;
    bool a_nonpos = true;
    int64_t d = 0;
    bool dv = false;

    for (int it = 0;; ++it) {
        const int st = it % ST;
        // full: the TMA bytes of this stage have landed (acquire for the async-proxy writes);
        // conv: the helper has written the float32 B / C copies
        mbar_wait(&s.full[st], (unsigned)(it / ST) & 1u, p.err);
        mbar_wait(&s.conv[st], (unsigned)(it / ST) & 1u, p.err);
        const int unit = s.unit[st];
        if (unit < 0) break;
        const int tile = s.tile[st];
        const int b = unit / p.nblk, blk = unit % p.nblk;
        const int t0 = (s.first[st] + tile) * PF_LT;
        const int rin = s.rin[st], rout = s.rout[st];
        const bool last = tile == s.ntl[st] - 1;

        if (tile == 0) {  // unit start: parameters and incoming state (staged by the producer)
            d = (int64_t)blk * PF_CPB + ch;
            dv = d < p.D;
            bool nonpos = true;
#pragma unroll
            for (int j = 0; j < PF_NP; ++j) {
                A2v[j].x = dv ? to_f(s.At[st][ch][n0 + 2 * j]) * LOG2E : 0.f;
                A2v[j].y = dv ? to_f(s.At[st][ch][n0 + 2 * j + 1]) * LOG2E : 0.f;
                nonpos = nonpos && A2v[j].x <= 0.f && A2v[j].y <= 0.f;
            }
            a_nonpos = __all_sync(FULL, nonpos);
            Dd = dv ? to_f(s.Dt[st][ch]) : 0.f;
            if (rin < 0) {   // the chain's start, or a state-only segment (from zero)
                sumd = 0.f;
#pragma unroll
                for (int j = 0; j < PF_NP; ++j) h2[j] = make_float2(0.f, 0.f);
                if (rin == RIN_START && p.h_prev != nullptr && dv) {
#pragma unroll
                    for (int j = 0; j < PF_NP; ++j)
                        h2[j] = make_float2(to_f(s.Ht[st][ch][n0 + 2 * j]), to_f(s.Ht[st][ch][n0 + 2 * j + 1]));
                }
            } else {
                const float* hs = &s.hin[st][ch * (NSTATE + 1)];
#pragma unroll
                for (int j = 0; j < PF_NP; ++j) h2[j] = make_float2(hs[n0 + 2 * j], hs[n0 + 2 * j + 1]);
                sumd = hs[NSTATE];
            }
        }

        const float* Bf = HALF ? &s.Bf[HALF ? st : 0][0][0] : reinterpret_cast<const float*>(&s.Bt[st][0][0]);
        const float* Cf = HALF ? &s.Cf[HALF ? st : 0][0][0] : reinterpret_cast<const float*>(&s.Ct[st][0][0]);
        const int yb = it & 1;
        if (p.has_out) mbar_wait(&s.yempty[yb], ((unsigned)(it / 2) & 1u) ^ 1u, p.err);

        // The tile's steps; CLAMP is uniform per tile (A <= 0 for the unit and no negative
        // delta in the tile make the clamp the identity), so each copy of the loop is
        // branch-free.
        // The tile's steps as 16-step chunks of two 8-step blocks (a checkpoint after each
        // chunk). CLAMP and HAS_OUT are uniform (CLAMP per tile: A <= 0 for the unit and no
        // negative delta in the tile make the clamp the identity), so each copy of the loop
        // is branch-free.
        const bool want_ck = p.ckpt != nullptr;
        // delta prefix record of the tile (launches with decay): the prefix before the tile and
        // the minimum over its steps of the prefix through each step
        float cstart = 0.f, cmin = 0.f;
        if constexpr (DECAY) {
            cstart = sumd;
            cmin = INFINITY;
        }
        auto run_tile = [&](auto clamp_tag, auto out_tag) {
            constexpr bool CLAMP = decltype(clamp_tag)::value;
            constexpr bool HAS_OUT = decltype(out_tag)::value;
#pragma unroll 1
            for (int c0 = 0; c0 < PF_LT; c0 += CK) {
#pragma unroll
                for (int i0 = c0; i0 < c0 + CK; i0 += 8) {
                    float dtv[8], uv[8], yv[8];
#pragma unroll
                    for (int r = 0; r < 8; ++r) {
                        dtv[r] = to_f(s.d[st][i0 + r][ch]);
                        uv[r] = to_f(s.u[st][i0 + r][ch]);
                        if constexpr (DECAY) {
                            sumd += dtv[r];
                            cmin = fminf(cmin, sumd);
                        }
                    }
                    fwd_block8<CLAMP>(h2, A2v, dtv, uv, Bf + i0 * NSTATE, Cf + i0 * NSTATE, n0, yv);
                    if constexpr (HAS_OUT && PF_LPC == 2) {
                        // the two lanes of a channel finish half the block's steps each (a
                        // reduce-scatter): lane half 0 steps 0-3, half 1 steps 4-7; the sums
                        // are the same as one full exchange per step (a + b = b + a)
                        const bool up = half != 0;
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const float send = up ? yv[j] : yv[j + 4];
                            const float keep = up ? yv[j + 4] : yv[j];
                            const float y = keep + __shfl_xor_sync(FULL, send, 1);
                            const float ur = up ? uv[j + 4] : uv[j];
                            s.y[yb][i0 + j + 4 * half][ch] = from_f<T>(fmaf(Dd, ur, y));
                        }
                    } else if constexpr (HAS_OUT) {
#pragma unroll
                        for (int r = 0; r < 8; ++r) {
                            float y = yv[r];
#pragma unroll
                            for (int o = 1; o < PF_LPC; o <<= 1) y += __shfl_xor_sync(FULL, y, o);
                            if (half == 0) s.y[yb][i0 + r][ch] = from_f<T>(fmaf(Dd, uv[r], y));
                        }
                    }
                }
                const int64_t kk = (int64_t)(t0 + c0) / CK;
                if (want_ck && kk < p.nck && dv) {
                    float4* cp = reinterpret_cast<float4*>(
                        p.ckpt + (((int64_t)b * p.nck + kk) * p.D + d) * NSTATE + n0);
#pragma unroll
                    for (int q = 0; q < PF_NP / 2; ++q)
                        cp[q] = make_float4(h2[2 * q].x, h2[2 * q].y, h2[2 * q + 1].x, h2[2 * q + 1].y);
                }
            }
        };
        const bool clamp = !(a_nonpos && s.dpos[st] != 0);
        if (p.has_out) {
            if (clamp) run_tile(std::true_type{}, std::true_type{});
            else run_tile(std::false_type{}, std::true_type{});
        } else {
            if (clamp) run_tile(std::true_type{}, std::false_type{});
            else run_tile(std::false_type{}, std::false_type{});
        }
        if constexpr (DECAY) {
            if (p.dpre != nullptr && half == 0 && dv)
                *reinterpret_cast<float2*>(p.dpre + (((int64_t)b * p.ntiles + t0 / PF_LT) * p.D + d) * 2) =
                    make_float2(cstart, cmin);
        }
        // this warp is done with the stage's inputs and with its rows of the y tile
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.empty[st]);
        if (p.has_out) {
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.yfull[yb]);
        }

        if (last) {
            if (rout >= 0) {   // a record for the unit that continues the chain
                float* hs = p.hand + (int64_t)rout * PF_HAND + ch * (NSTATE + 1);
#pragma unroll
                for (int j = 0; j < PF_NP; ++j) {
                    hs[n0 + 2 * j] = h2[j].x;
                    hs[n0 + 2 * j + 1] = h2[j].y;
                }
                if (half == 0) hs[NSTATE] = sumd;
                if (p.mode == 0) {
                    __threadfence();
                    __syncwarp();
                    if (lane == 0) atomicAdd(&p.flags[rout], 1);
                }
            } else if (rout == ROUT_END && dv) {
                if (p.h_last != nullptr) {
                    T* hl = static_cast<T*>(p.h_last) + ((int64_t)b * p.D + d) * NSTATE + n0;
#pragma unroll
                    for (int j = 0; j < PF_NP; ++j) {
                        hl[2 * j] = from_f<T>(h2[j].x);
                        hl[2 * j + 1] = from_f<T>(h2[j].y);
                    }
                }
                if (p.decay != nullptr) {
                    float* dc = p.decay + ((int64_t)b * p.D + d) * NSTATE + n0;
#pragma unroll
                    for (int j = 0; j < PF_NP; ++j) {
                        dc[2 * j] = ex2(fminf(A2v[j].x * sumd, ARG2_HI));
                        dc[2 * j + 1] = ex2(fminf(A2v[j].y * sumd, ARG2_HI));
                    }
                }
            }
        }
    }
}

// Fold of the state-only pass's records (few chains, K independent segments per chain).
// For chain c and (channel, state), record k holds segment k's end state from its own start
// (segment 0 from h_prev, the others from zero) and its delta sum; afterwards it holds the
// true state after segment k and the delta sum from the sequence start:
//   h_k = 2^(A*log2(e) * sumd_k) h_{k-1} + R_k,   S_k = S_{k-1} + sumd_k
// A segment's decay is the product of its per-step factors, exp(A * sum delta); the clamp is
// the per-step one applied to the sum, the identity for A <= 0 and delta >= 0.
template <typename T>
__global__ void ss_fwd_fold_kernel(float* __restrict__ hand, const T* __restrict__ A, int nblk,
                                   int nchains, int K, int D) {
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;   // (c, ch, n), n fastest
    if (tid >= (int64_t)nchains * PF_CPB * NSTATE) return;   // whole warps: the count is a multiple of 2048
    const int n = (int)(tid % NSTATE);
    const int ch = (int)((tid / NSTATE) % PF_CPB);
    const int c = (int)(tid / (NSTATE * PF_CPB));
    const int64_t d = (int64_t)(c % nblk) * PF_CPB + ch;
    const float a2 = d < D ? to_f(A[d * NSTATE + n]) * LOG2E : 0.f;
    float* r = hand + (int64_t)c * K * PF_HAND + ch * (NSTATE + 1);
    float h = r[n], S = r[NSTATE];
    for (int k = 1; k < K - 1; ++k) {
        float* rk = r + (int64_t)k * PF_HAND;
        const float sk = rk[NSTATE];
        h = fmaf(ex2(fminf(a2 * sk, ARG2_HI)), h, rk[n]);
        S += sk;
        rk[n] = h;
        __syncwarp();   // every state of the channel has read rk[NSTATE]
        if (n == 0) rk[NSTATE] = S;
    }
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
    const size_t es = dtype == 0 ? 4 : 2;
    cuuint64_t dims[3] = {(cuuint64_t)W, (cuuint64_t)L, (cuuint64_t)B};
    cuuint64_t strides[2] = {(cuuint64_t)(W * es), (cuuint64_t)(W * L * es)};
    cuuint32_t box[3] = {(cuuint32_t)bw, (cuuint32_t)bl, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, dtype == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                         : dtype == 1 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
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
    pl.ok = num_sms > 0 && pl.nchains >= num_sms;
    if (!pl.ok) return pl;
    // one run of the concatenated tiles per SM (seg_tiles: the longest run); K = 2 when a
    // run boundary cuts a chain (a chain is cut at most once: runs are >= one chain long)
    pl.grid = num_sms;
    const int64_t T = (int64_t)pl.nchains * pl.ntiles;
    pl.seg_tiles = (int)((T + pl.grid - 1) / pl.grid);
    pl.K = 1;
    for (int r = 1; r < pl.grid; ++r)
        if ((T * r / pl.grid) % pl.ntiles != 0) {
            pl.K = 2;
            break;
        }
    return pl;
}

int pick_split_segments(int nchains, int ntiles, int num_sms, int min_seg_tiles) {
    // time ~ waves x segment length (units of one pass run in parallel); the small term per
    // segment stands for the records, the fold and each unit's start-up
    int best_k = 0;
    double best = 1e300;
    for (int K = 2; K <= ntiles / min_seg_tiles; ++K) {
        const int seg = (ntiles + K - 1) / K;
        if ((ntiles + seg - 1) / seg != K) continue;
        const int64_t U = (int64_t)nchains * K;
        const int64_t waves = (U + num_sms - 1) / num_sms;
        const double cost = (double)waves * seg + 0.02 * K;
        if (cost < best - 1e-9) {
            best = cost;
            best_k = K;
        }
    }
    return best_k;
}

PersistPlan plan_persistent_split(int64_t B, int64_t L, int64_t D, int num_sms) {
    PersistPlan pl{};
    pl.nblk = (int)((D + PF_CPB - 1) / PF_CPB);
    pl.nchains = (int)(B * pl.nblk);
    pl.ntiles = (int)((L + PF_LT - 1) / PF_LT);
    pl.ok = false;
    // below ~512 steps one generic pass is as fast as three short launches
    if (pl.nchains <= 0 || pl.nchains >= num_sms || (int64_t)pl.ntiles * PF_LT < 512) return pl;
    const int K = pick_split_segments(pl.nchains, pl.ntiles, num_sms, MWC_FWD_SPLIT_MIN_SEG_TILES);
    if (K < 2) return pl;
    pl.K = K;
    pl.seg_tiles = (pl.ntiles + K - 1) / K;
    pl.grid = (int)std::min<int64_t>(num_sms, (int64_t)pl.nchains * pl.K);
    pl.ok = true;
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

template <typename T, bool DECAY>
static cudaError_t launch_pf_t(const PFwdArgs& a, int grid, cudaStream_t s) {
    const size_t smem = sizeof(PFwdSmem<T>);
    cudaError_t e = ensure_smem_attr<ss_fwd_persistent_kernel<T, DECAY>>((int)smem);
    if (e != cudaSuccess) return e;
    ss_fwd_persistent_kernel<T, DECAY><<<grid, PF_NT, smem, s>>>(a);
    return cudaGetLastError();
}

template <typename T>
static cudaError_t launch_pf(const PFwdArgs& a, int grid, cudaStream_t s) {
    return a.decay != nullptr ? launch_pf_t<T, true>(a, grid, s) : launch_pf_t<T, false>(a, grid, s);
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
    if (dtype == 2) return launch_pf<__nv_bfloat16>(a, pl.grid, s);
    return dtype == 1 ? launch_pf<__half>(a, pl.grid, s) : launch_pf<float>(a, pl.grid, s);
}

// Few chains: pass 1 scans segments 0..K-2 for their end states only (delta sums always
// on, no outputs), the fold turns the records into each segment's incoming state, and pass 2
// runs the full scan with every segment seeded from its record. Each pass has its own unit
// counter in the header, which is cleared once.
cudaError_t launch_fwd_persistent_split(PFwdArgs& a, const PersistPlan& pl, int dtype, void* ws,
                                        cudaStream_t s) {
    char* w = static_cast<char*>(ws);
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
    PFwdArgs p1 = a;
    p1.mode = 1;
    p1.counter = reinterpret_cast<int*>(w);
    p1.has_out = 0;
    p1.ckpt = nullptr;
    p1.h_last = nullptr;
    p1.decay = nullptr;
    p1.dpre = nullptr;   // state-only segments sum delta from their own start
    const int grid1 = (int)std::min<int64_t>(pl.grid, (int64_t)pl.nchains * (pl.K - 1));
    e = dtype == 2 ? launch_pf_t<__nv_bfloat16, true>(p1, grid1, s)
      : dtype == 1 ? launch_pf_t<__half, true>(p1, grid1, s)
                   : launch_pf_t<float, true>(p1, grid1, s);
    if (e != cudaSuccess) return e;
    const int64_t nthr = (int64_t)pl.nchains * PF_CPB * NSTATE;
    const unsigned fb = (unsigned)((nthr + 255) / 256);
    if (dtype == 2)
        ss_fwd_fold_kernel<__nv_bfloat16><<<fb, 256, 0, s>>>(a.hand, static_cast<const __nv_bfloat16*>(a.A),
                                                             pl.nblk, pl.nchains, pl.K, a.D);
    else if (dtype == 1)
        ss_fwd_fold_kernel<__half><<<fb, 256, 0, s>>>(a.hand, static_cast<const __half*>(a.A), pl.nblk,
                                                      pl.nchains, pl.K, a.D);
    else
        ss_fwd_fold_kernel<float><<<fb, 256, 0, s>>>(a.hand, static_cast<const float*>(a.A), pl.nblk,
                                                     pl.nchains, pl.K, a.D);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    a.mode = 2;
    a.counter = reinterpret_cast<int*>(w + 8);
    if (dtype == 2) return launch_pf<__nv_bfloat16>(a, pl.grid, s);
    return dtype == 1 ? launch_pf<__half>(a, pl.grid, s) : launch_pf<float>(a, pl.grid, s);
}

}  // namespace mwc
