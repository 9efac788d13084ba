// gw_gemv.cu — decode expert GEMVs (gate_up + activation, down x routing
// weight) over the HBM-resident bank.
//
// The reference evaluates each routed (expert, token) pair as
// mxfp4_gemv_bias -> gptoss_expert_activation / expert_activation_swiglu ->
// mxfp4_gemv_bias -> expert_accumulate (Metal/MoE/expert.metal:46-116,
// :380-393; ExpertRunner.applyAssignments, Runtime/ExpertRunner.swift:108-183),
// each block of 32 products summed in fp32 and then multiplied by the
// block's E8M0 scale (Metal/Quant/dequant_gemv.metal:50-63).  This kernel does
// the same arithmetic for every token routed to an expert from one pass over
// the expert's weights.
//
// Layout and data movement.  The bank stores each MXFP4 matrix in 16-row
// tiles, each tile in groups of eight 32-column blocks, a group's 16 rows x
// 128 bytes row-major (2 KB; the last group of a row narrower when K/32 is not
// a multiple of 8).  A CTA has kEW consumer warps, each owning kNT tiles (or
// a K-split share of them), and one producer warp.  Per stage the producer
// issues one TMA box that holds the same group of all the CTA's tiles (48 KB,
// 128-byte swizzle, so the consumers' reads are free of bank conflicts) and
// one box of their scale bytes, into a kEStages-deep ring of stages guarded
// by full / empty mbarriers; the consumers only wait, compute and release.
// The tokens' f16 rows are staged once per pass of up to four tokens, laid
// out as the MMA's B fragments.
//
// Arithmetic.  mma.sync.m16n8k16 (f16 x f16 -> fp32) with the 16 weight rows
// as M.  Thread (g, t) feeds K-columns 8t..8t+7 of each 32-column block —
// byte t*4..t*4+3 of each of its two rows, widened with cvt.rn.f16x2.e2m1x2 —
// so one MMA pair covers exactly one block and the B fragment is one 16-byte
// shared load.  The 8 N-columns hold (block slot, token): 8 blocks x 1
// token, 4 x 2 or 2 x 4 (by the pass's token count), the B operand of a
// column being zero outside its block slot; after each window of blocks the
// fp32 partials are multiplied by their block's scale into fp32 accumulators
// (the reference's `acc += partial * scale`).
//
// Every wait on an mbarrier is bounded (~2 s); a wait that runs out sets a
// bit in the status word, the CTA stops computing but keeps its barrier
// protocol, and the producer waits (bounded) for the copies it has in flight
// before the CTA exits.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <algorithm>

#include "gw_async.cuh"
#include "gw_device.cuh"
#include "gw_internal.h"

namespace gw {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();  // gw_grouped.cu

namespace {

constexpr int kEW = 24;                      // consumer warps per CTA (one CTA per SM)
constexpr int kNT = 1;                       // tiles per consumer warp
constexpr int kCT = kEW * kNT;               // tiles per stage (per round)
constexpr int kBoxT = 6;                     // tiles per TMA box of weights (divides kCT / 4)
constexpr int kEThreads = (kEW + 1) * 32;    // + the producer warp
constexpr int kEStages = 3;                  // stages in flight per CTA
constexpr int kEPass = kGemvPass;            // tokens per pass over the weights
constexpr int kGrp = 2048;                   // one tile's full group: 16 rows x 128 bytes
constexpr int kGrpSc = 128;                  // its scale bytes
constexpr int kStageW = kCT * kGrp;          // 48 KB of weights per stage
constexpr int kStageS = kCT * kGrpSc;        // 3 KB of scales per stage
constexpr unsigned kStatusGemv = 0x200u;
// try_wait suspends the waiting threads up to this long (they wake as soon as
// the phase completes).
constexpr uint32_t kSuspendNs = 100000;

struct ExpertGemvArgs {
    const uint8_t* base;   // local expert 0 of the layer
    int64_t stride;        // bytes per expert
    int64_t off_bias;
    int M, K;              // matrix rows, columns
    int ksplit;            // K-splits (tiles per split = kCT / ksplit)
    int k, shard_count;
    int F, H;
    float limit, alpha;
    MoeWork w;
};

// The four TMA views of one matrix of the layer's bank (see launch_expert_gemv).
struct GemvMaps {
    CUtensorMap w_full, w_narrow, s_full, s_narrow;
};

// Shared-memory carve-up (dynamic; the base is aligned to 1024 for the
// 128-byte swizzle).  The staged tokens are laid out for the MMA's B operand
// directly: entry (group, block j, column g) is the 64 bytes lane group g
// reads for block j — the block of x of the column's token when the column's
// block slot is j's, else zeros — so no lane selects between x and zero.
struct SmemPlan {
    int ring, sc, xe, red, bars, total;
};

__host__ __device__ inline SmemPlan smem_plan(int K) {
    const int ngrp = (K / 32 + 7) / 8;
    SmemPlan p;
    p.ring = 0;
    p.sc = p.ring + kEStages * kStageW;
    p.xe = p.sc + kEStages * kStageS;
    p.red = p.xe + ngrp * 8 * 8 * 64;
    p.bars = p.red + kCT * 2 * 8 * kEPass * 4;
    p.total = p.bars + 2 * kEStages * 8 + 16 + 1024;  // + abort flag, alignment slack
    return p;
}

// Shared-memory reads as plain C++ loads (the compiler schedules them; the
// barrier waits' "memory" clobbers keep them after the data has landed).
__device__ __forceinline__ uint32_t ld32(const unsigned char* p) { return *reinterpret_cast<const uint32_t*>(p); }
__device__ __forceinline__ uint4 ld128(const unsigned char* p) { return *reinterpret_cast<const uint4*>(p); }

// One 5-D tile of `map` at (0, 0, c2, c3, c4) -> shared, counted on `bar`.
__device__ __forceinline__ void tma_5d(uint32_t dst, const CUtensorMap* map, int c2, int c3, int c4,
                                       uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %2, "
        "%3, %4, %5}], [%6];" ::"r"(dst),
        "l"(map), "r"(0), "r"(c2), "r"(c3), "r"(c4), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void arrive_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool try_parity(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(kSuspendNs)
        : "memory");
    return ok != 0;
}
// Bounded wait on a phase; false once it ran out (status bit set).
__device__ __forceinline__ bool wait_parity(uint32_t bar, uint32_t parity, unsigned* status) {
    if (try_parity(bar, parity)) return true;
    const long long t0 = clock64();
    for (uint32_t i = 1;; ++i) {
        if (try_parity(bar, parity)) return true;
        if ((i & 63) == 0 && clock64() - t0 > kWaitCycles) {
            if (status) atomicOr(status, kStatusGemv);
            return false;
        }
    }
}


// d = A B (the accumulator starts from zero)
__device__ __forceinline__ void mma_f16_z(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %10, %10, %10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
}
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float e8m0(uint32_t byte) { return __uint_as_float(byte << 23); }  // gemv_scale

// One group of kNT tiles of one warp: w blocks (w = 8 for full,
// 128-byte-swizzled groups, else narrow unswizzled ones); tile rows g and
// g + 8 as the MMA's rows g / g + 8, kTok tokens per MMA (8 / kTok block
// slots).  A: the first tile's group in shared memory (the next tile's
// follows `astep` bytes later), Sc: its 16 x w scale bytes (next tile's
// `sstep` later); off[j] = (j ^ g) * 16, the swizzled position of block j in
// rows g and g + 8 (both have row % 8 = g); xg: this lane's B entries of the
// group (entry (j, g), quarter t), shared by the tiles.  Accumulates
// acc[tile][row][column of the lane].
template <int kTok, bool kFull>
__device__ __forceinline__ void group_mma(const unsigned char* A, int astep, const unsigned char* Sc, int sstep,
                                          int w, int g, int t, const uint32_t (&off)[8], const unsigned char* xg,
                                          float (&acc)[kNT][2][2]) {
    constexpr int kBlk = 8 / kTok;
    const int wl = kFull ? 8 : w;
    const int sw = kFull ? 8 : w;  // scale bytes per row
    auto scale = [&](int ti, int row, int i) -> float {
        return (kFull || i < wl) ? e8m0(Sc[ti * sstep + row * sw + i]) : 0.f;
    };
    const unsigned char* rowA = A + (kFull ? g * 128 : g * 16 * w) + 4 * t;
    const int rowB = kFull ? 8 * 128 : 8 * 16 * w;  // row g + 8, relative to row g
    // one accumulator per tile: the block's second MMA adds into its first's
    // result (the pair's partial sums are then one register, not two to add)
    float d[kNT][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        if (!kFull && j % kBlk == 0) {  // a narrow group may end before its window does
#pragma unroll
            for (int ti = 0; ti < kNT; ++ti)
#pragma unroll
                for (int q = 0; q < 4; ++q) d[ti][q] = 0.f;
        }
        if (kFull || j < wl) {
            const uint4 xv = ld128(xg + j * 512);
#pragma unroll
            for (int ti = 0; ti < kNT; ++ti) {
                const unsigned char* pa = rowA + ti * astep + (kFull ? off[j] : j * 16);
                const uint32_t wa = ld32(pa);
                const uint32_t wb = ld32(pa + rowB);
                uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
                e2m1x8_to_f16x8(wa, a0, a1, a2, a3);
                e2m1x8_to_f16x8(wb, b0, b1, b2, b3);
                if (kFull && j % kBlk == 0)  // the window's first block starts the accumulator
                    mma_f16_z(d[ti], a0, b0, a1, b1, xv.x, xv.y);
                else
                    mma_f16(d[ti], a0, b0, a1, b1, xv.x, xv.y);
                mma_f16(d[ti], a2, b2, a3, b3, xv.z, xv.w);
            }
        }
        if (j % kBlk == kBlk - 1) {  // flush the window of blocks [j - kBlk + 1, j]
            const int jb = j - kBlk + 1;
#pragma unroll
            for (int ti = 0; ti < kNT; ++ti) {
                if (kTok == 1) {  // columns 2t, 2t + 1 = blocks 2t, 2t + 1
                    acc[ti][0][0] = fmaf(d[ti][0], scale(ti, g, 2 * t), acc[ti][0][0]);
                    acc[ti][0][0] = fmaf(d[ti][1], scale(ti, g, 2 * t + 1), acc[ti][0][0]);
                    acc[ti][1][0] = fmaf(d[ti][2], scale(ti, g + 8, 2 * t), acc[ti][1][0]);
                    acc[ti][1][0] = fmaf(d[ti][3], scale(ti, g + 8, 2 * t + 1), acc[ti][1][0]);
                } else {  // columns 2t, 2t + 1 share one block
                    const int bi = jb + (kTok == 2 ? t : kTok == 4 ? (t >> 1) : 0);
                    const float fa = scale(ti, g, bi), fb = scale(ti, g + 8, bi);
                    acc[ti][0][0] = fmaf(d[ti][0], fa, acc[ti][0][0]);
                    acc[ti][0][1] = fmaf(d[ti][1], fa, acc[ti][0][1]);
                    acc[ti][1][0] = fmaf(d[ti][2], fb, acc[ti][1][0]);
                    acc[ti][1][1] = fmaf(d[ti][3], fb, acc[ti][1][1]);
                }
            }
        }
    }
}

// True on one lane of the (converged) warp.
__device__ __forceinline__ bool elect_one() {
    uint32_t pred;
    asm volatile(
        "{\n\t.reg .pred P;\n\telect.sync _|P, 0xffffffff;\n\tselp.u32 %0, 1, 0, P;\n\t}"
        : "=r"(pred));
    return pred != 0;
}
__device__ __forceinline__ void arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// the kEW consumer warps only
__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kEW * 32) : "memory"); }
// the same barrier, returning whether any consumer thread passed true
__device__ __forceinline__ bool consumers_sync_or(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %1, 0;\n\tbar.red.or.pred p, 1, %2, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "n"(kEW * 32)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ void tma_4d(uint32_t dst, const CUtensorMap* map, int c1, int c2, int c3, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
        "%4, %5}], [%6];" ::"r"(dst),
        "l"(map), "r"(0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void tma_3d(uint32_t dst, const CUtensorMap* map, int c1, int c2, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
        "%4}], [%5];" ::"r"(dst),
        "l"(map), "r"(0), "r"(c1), "r"(c2), "r"(bar)
        : "memory");
}

// kMode 0 / 1: gate_up with the clamped GLU / SiLU epilogue (f16 activations
// per slot); 2: down x routing weight (fp32 per slot).
//
// Persistent: `gridDim.x` CTAs (at most one per SM) share the layer's work
// items — item i = (active expert i / ny, tile round i % ny), a round being
// kCT / ksplit tiles over the whole K range — through the self-resetting
// counter pair a.w.sched (next item, CTAs finished).  The producer warp takes
// the next item as soon as it has issued the last stage of the current one,
// so the weight stream of an SM runs on across items while the consumers
// finish one item's epilogue and stage the next item's tokens.  Each stage
// carries its item id in shared memory; item -1 ends the consumers' loop.
template <int kMode>
__global__ void __launch_bounds__(kEThreads, 1) k_expert_gemv(const __grid_constant__ GemvMaps maps,
                                                              ExpertGemvArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const SmemPlan P = smem_plan(a.K);
    const uint32_t sbase = (saddr(smem_raw) + 1023u) & ~1023u;
    unsigned char* sgen = smem_raw + (sbase - saddr(smem_raw));
    __shared__ int meta_row[kEPass], meta_slot[kEPass];
    __shared__ float meta_mul[kEPass];
    __shared__ int stage_item[kEStages];

    // the warp index through a shuffle: the compiler then knows every value
    // derived from it is warp-uniform
    const int warp = __shfl_sync(0xffffffffu, (int)(threadIdx.x >> 5), 0);
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int nblk = a.K >> 5, nfull = nblk >> 3, ngrp = (nblk + 7) >> 3;
    const int wlast = nblk - 8 * (ngrp - 1);
    const int ntiles = a.M >> 4;
    const int ks = a.ksplit, tb = kCT / ks;  // tiles per split and item
    const int per = (ngrp + ks - 1) / ks;    // stages per pass
    const int ny = (ntiles + tb - 1) / tb;   // items per expert
    unsigned* status = a.w.status;
    const uint32_t fullb = sbase + P.bars, emptyb = fullb + kEStages * 8;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(sgen + P.bars + 2 * kEStages * 8);

    if (threadIdx.x < kEStages) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(fullb + threadIdx.x * 8) : "memory");
        asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(emptyb + threadIdx.x * 8), "n"(kEW) : "memory");
    }
    if (threadIdx.x == 0) *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    __syncthreads();

    if (warp == kEW) {
        // ---- producer: stages of an item = steps s; split sp's group
        // sp * per + s of the item's tiles
        if (elect_one()) {
            // a wait of this launch (or an earlier one since the last gw_sync)
            // ran out: the results are already invalid, so take no work
            const bool dead = status && (*(volatile unsigned*)status & kStatusGemv);
            const int na = *a.w.nactive;
            const int nitems = dead ? 0 : (na + *a.w.nextra) * ny;
            int slot = 0;
            uint32_t phase = 0;
            long long it = 0;  // stages issued
            bool ok = true;
            auto acquire = [&]() {  // the next ring slot is free (bounded wait)
                if (it >= kEStages && ok) {
                    ok = wait_parity(emptyb + slot * 8, phase ^ 1, status);
                    if (!ok) *abort_flag = 1;
                }
                if (ok && *abort_flag) ok = false;
                return ok;
            };
            // the first item is the CTA's own; later ones come from the counter,
            // requested while the current item's first stage is in flight
            int item = blockIdx.x;
            while (item < nitems) {
                const int q = item / ny;
                const int e = q < na ? a.w.active[q] : (a.w.extra[q - na] & 0xFFFF);
                const int le = e / a.shard_count;
                const int tt = (item % ny) * tb;
                int next = nitems;
                for (int i = 0, s = 0; i < per; ++i) {
                    if (!acquire()) break;
                    uint32_t bytes = 0;
                    for (int sp = 0; sp < ks; ++sp) {
                        const int grp = sp * per + s;
                        if (grp >= min(ngrp, (sp + 1) * per)) continue;
                        bytes += grp < nfull ? (uint32_t)tb * (kGrp + kGrpSc) : (uint32_t)tb * 17u * 16u * wlast;
                    }
                    stage_item[slot] = item;
                    const uint32_t bar = fullb + slot * 8;
                    arrive_tx(bar, bytes);
                    for (int sp = 0; sp < ks; ++sp) {
                        const int grp = sp * per + s;
                        if (grp >= min(ngrp, (sp + 1) * per)) continue;
                        const uint32_t wdst = sbase + P.ring + slot * kStageW;
                        const uint32_t sdst = sbase + P.sc + slot * kStageS;
                        if (grp < nfull) {
                            for (int b = 0; b < tb; b += kBoxT)
                                tma_5d(wdst + (sp * tb + b) * kGrp, &maps.w_full, grp, tt + b, le, bar);
                            tma_4d(sdst + sp * tb * kGrpSc, &maps.s_full, grp, tt, le, bar);
                        } else {
                            for (int b = 0; b < tb; b += kBoxT)
                                tma_4d(wdst + sp * tb * kGrp + b * 256 * wlast, &maps.w_narrow, 0, tt + b, le, bar);
                            tma_3d(sdst + sp * tb * kGrpSc, &maps.s_narrow, tt, le, bar);
                        }
                    }
                    if (i == 0) next = (int)gridDim.x + (int)atomicAdd(&a.w.sched[0], 1u);
                    if (++s == per) s = 0;
                    ++it;
                    if (++slot == kEStages) { slot = 0; phase ^= 1; }
                }
                if (!ok) break;
                item = next;
            }
            // end of work: a stage without copies whose item id is -1
            if (acquire()) {
                stage_item[slot] = -1;
                arrive(fullb + slot * 8);
            } else {
                // after a wait ran out: let the copies still in flight land
                for (long long j = it - kEStages > 0 ? it - kEStages : 0; j < it; ++j)
                    (void)wait_parity(fullb + (j % kEStages) * 8, (uint32_t)((j / kEStages) & 1), nullptr);
            }
        }
        __syncwarp();
    } else {
        // ---- consumers: warp = (split sp, position wl); its kNT tiles of an
        // item are tiles wl * kNT .. + kNT - 1 of the split's tb
        const int wps = kEW / ks;  // consumer warps per split
        const int sp = warp / wps, wl = warp % wps;
        const int g0 = min(ngrp, sp * per), g1 = min(ngrp, g0 + per);
        const bool leader = elect_one();
        // this lane reads tile rows g and g + 8 (the eight rows a quad phase
        // reads sit on distinct 128-byte-swizzle chunks); block j of both is
        // at 16 (j ^ g) in its row
        uint32_t off[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) off[j] = (uint32_t)((j ^ g) << 4);
        const __half* xsrc = kMode == 2 ? a.w.act : a.w.x16;
        const unsigned char* xg0 = sgen + P.xe + g * 64 + 16 * t;
        float* red = reinterpret_cast<float*>(sgen + P.red);
        bool ok = true;
        int slot = 0;
        uint32_t phase = 0;
        auto wait_full = [&]() {  // this warp's bounded wait on the current stage
            if (ok) {
                ok = try_parity(fullb + slot * 8, phase) || wait_parity(fullb + slot * 8, phase, status);
                if (!ok) *abort_flag = 1;
            }
            ok = __all_sync(0xffffffffu, ok) && !*abort_flag;
            return ok;
        };
        // Every consumer warp runs the same sequence of consumer barriers: the
        // decisions to stop (end of work, or a wait that ran out anywhere in
        // the CTA) are taken at a barrier with an OR over all consumers.
        const int na = *a.w.nactive;
        for (;;) {
            // (also: the previous item's staged x, results and metadata are consumed)
            const bool here = wait_full();
            if (consumers_sync_or(!here)) break;
            const int item = stage_item[slot];
            if (item < 0) break;
            // item -> (expert, pass of up to kEPass of its tokens, tile round)
            const int q = item / ny;
            const int ex = q < na ? 0 : a.w.extra[q - na];
            const int e = q < na ? a.w.active[q] : (ex & 0xFFFF);
            const int c0 = (ex >> 16) * kEPass;
            const int n = min(kEPass, min(a.w.counts[e], a.w.tcap) - c0);
            const int* list = a.w.lists + (int64_t)e * a.w.tcap;
            const int le = e / a.shard_count;
            const int tile0 = (item % ny) * tb;
            const bool any = tile0 + wl * kNT < ntiles;  // the warp's first tile exists
            // the bias pair each emitting lane adds (gate_up: rows 2f, 2f + 1 of
            // feature f = tile * 8 + g; down: rows tile * 16 + g, + 8), loaded
            // now so its latency hides behind the stage loop
            float bias0[kNT], bias1[kNT];
            {
                const uint16_t* bias =
                    reinterpret_cast<const uint16_t*>(a.base + (int64_t)le * a.stride + a.off_bias);
#pragma unroll
                for (int ti = 0; ti < kNT; ++ti) {
                    const int tile = tile0 + wl * kNT + ti;
                    bias0[ti] = bias1[ti] = 0.f;
                    if (sp == 0 && tile < ntiles) {
                        const int i0 = kMode == 2 ? tile * 16 + g : 2 * (tile * 8 + g);
                        const int i1 = kMode == 2 ? i0 + 8 : i0 + 1;
                        bias0[ti] = bf16_bits_to_f32(__ldg(bias + i0));
                        bias1[ti] = bf16_bits_to_f32(__ldg(bias + i1));
                    }
                }
            }
            {
                if (threadIdx.x < n) {
                    const int sl = list[c0 + threadIdx.x];
                    const int row = kMode == 2 ? sl : sl / a.k;
                    meta_slot[threadIdx.x] = sl;
                    meta_row[threadIdx.x] = row;
                    meta_mul[threadIdx.x] = kMode == 2 ? a.w.weights[sl] : a.w.xmul[row];
                }
                consumers_sync();
                // B entries: quarter q of (group, block j, column c) <- x[token of c][block] or zeros
                for (int i = threadIdx.x; i < ngrp * 256; i += kEW * 32) {
                    const int q = i & 3, c = (i >> 2) & 7, j = (i >> 5) & 7, grp = i >> 8;
                    bool live;
                    int tok;
                    if (n == 1) { live = j == c; tok = 0; }
                    else if (n == 2) { live = (j & 3) == (c >> 1); tok = c & 1; }
                    else if (n <= 4) { live = (j & 1) == (c >> 2); tok = c & 3; }
                    else { live = true; tok = c; }
                    live = live && tok < n && grp * 8 + j < nblk;
                    uint4 v = make_uint4(0u, 0u, 0u, 0u);
                    if (live)
                        v = __ldg(reinterpret_cast<const uint4*>(xsrc + (int64_t)meta_row[tok] * a.K) + (grp * 8 + j) * 4 + q);
                    reinterpret_cast<uint4*>(sgen + P.xe)[i] = v;
                }
                consumers_sync();
                float acc[kNT][2][2];
#pragma unroll
                for (int ti = 0; ti < kNT; ++ti) acc[ti][0][0] = acc[ti][0][1] = acc[ti][1][0] = acc[ti][1][1] = 0.f;
                for (int s = 0; s < per; ++s) {
                    const int grp = g0 + s;
                    if (wait_full() && any && grp < g1) {
                        const unsigned char* xg = xg0 + grp * 4096;
                        const unsigned char* W = sgen + P.ring + slot * kStageW + sp * tb * kGrp;
                        const unsigned char* S = sgen + P.sc + slot * kStageS + sp * tb * kGrpSc;
                        if (grp < nfull) {
                            const unsigned char* A = W + wl * kNT * kGrp;
                            const unsigned char* Sc = S + wl * kNT * kGrpSc;
                            if (n == 1) group_mma<1, true>(A, kGrp, Sc, kGrpSc, 8, g, t, off, xg, acc);
                            else if (n == 2) group_mma<2, true>(A, kGrp, Sc, kGrpSc, 8, g, t, off, xg, acc);
                            else if (n <= 4) group_mma<4, true>(A, kGrp, Sc, kGrpSc, 8, g, t, off, xg, acc);
                            else group_mma<8, true>(A, kGrp, Sc, kGrpSc, 8, g, t, off, xg, acc);
                        } else {
                            const unsigned char* A = W + wl * kNT * 256 * wlast;
                            const unsigned char* Sc = S + wl * kNT * 16 * wlast;
                            const int as = 256 * wlast, ss = 16 * wlast;
                            if (n == 1) group_mma<1, false>(A, as, Sc, ss, wlast, g, t, off, xg, acc);
                            else if (n == 2) group_mma<2, false>(A, as, Sc, ss, wlast, g, t, off, xg, acc);
                            else if (n <= 4) group_mma<4, false>(A, as, Sc, ss, wlast, g, t, off, xg, acc);
                            else group_mma<8, false>(A, as, Sc, ss, wlast, g, t, off, xg, acc);
                        }
                    }
                    __syncwarp();
                    if (leader) arrive(emptyb + slot * 8);  // this warp is done with the stage
                    if (++slot == kEStages) { slot = 0; phase ^= 1; }
                }
#pragma unroll
                for (int ti = 0; ti < kNT; ++ti) {
                    const int tl = wl * kNT + ti;          // tile within the split
                    if (tile0 + tl >= ntiles) continue;
                    // columns -> (row, token): sum the block slots held by the quad
                    float v[2][2];
#pragma unroll
                    for (int rr = 0; rr < 2; ++rr) {
                        if (n == 1) {
                            float x = acc[ti][rr][0];
                            x += __shfl_xor_sync(0xffffffffu, x, 1);
                            x += __shfl_xor_sync(0xffffffffu, x, 2);
                            v[rr][0] = x;
                            v[rr][1] = 0.f;
                        } else if (n == 2) {
#pragma unroll
                            for (int c = 0; c < 2; ++c) {
                                float x = acc[ti][rr][c];
                                x += __shfl_xor_sync(0xffffffffu, x, 1);
                                x += __shfl_xor_sync(0xffffffffu, x, 2);
                                v[rr][c] = x;
                            }
                        } else if (n <= 4) {
#pragma unroll
                            for (int c = 0; c < 2; ++c)
                                v[rr][c] = acc[ti][rr][c] + __shfl_xor_sync(0xffffffffu, acc[ti][rr][c], 2);
                        } else {
                            v[rr][0] = acc[ti][rr][0];
                            v[rr][1] = acc[ti][rr][1];
                        }
                    }
                    // red[tile slot][r][g][token] = tile row 8r + g
                    float* rw = red + (sp * tb + tl) * (2 * 8 * kEPass);
                    const int tk = n <= 2 ? 0 : 2 * t;
                    if ((n <= 2 && t == 0) || (n > 2 && n <= 4 && t < 2) || n > 4) {
                        rw[0 * 8 * kEPass + g * kEPass + tk] = v[0][0];
                        rw[1 * 8 * kEPass + g * kEPass + tk] = v[1][0];
                        rw[0 * 8 * kEPass + g * kEPass + tk + 1] = v[0][1];
                        rw[1 * 8 * kEPass + g * kEPass + tk + 1] = v[1][1];
                    }
                }
                // a tile with K-split partials waits for all of them; a warp that
                // owns its tiles outright only for its own lanes
                if (ks > 1) consumers_sync();
                else __syncwarp();
                // split-0 warps emit their tiles: lane (g, t) -> tokens t, t + 4
                if (sp == 0 && ok) {
                    // gate_up: feature g = tile rows 2g (gate), 2g + 1 (up); down: rows g, g + 8
                    const int q0 = kMode == 2 ? g : 2 * g, q1 = kMode == 2 ? g + 8 : 2 * g + 1;
#pragma unroll
                    for (int half = 0; half < 2; ++half) {
                        const int tok = t + 4 * half;
                        if (tok >= n) break;
                        const int sl = meta_slot[tok];
                        const float mul = meta_mul[tok];
#pragma unroll
                        for (int ti = 0; ti < kNT; ++ti) {
                            const int tl = wl * kNT + ti;
                            const int tile = tile0 + tl;
                            if (tile >= ntiles) continue;
                            float y0 = 0.f, y1 = 0.f;
                            for (int q = 0; q < ks; ++q) {
                                const float* rw = red + (q * tb + tl) * (2 * 8 * kEPass);
                                y0 += rw[(q0 >> 3) * 8 * kEPass + (q0 & 7) * kEPass + tok];
                                y1 += rw[(q1 >> 3) * 8 * kEPass + (q1 & 7) * kEPass + tok];
                            }
                            if (kMode != 2) {
                                const int f = tile * 8 + g;
                                const float gate = y0 * mul + bias0[ti];
                                const float up = y1 * mul + bias1[ti];
                                a.w.act[(int64_t)sl * a.F + f] = __float2half_rn(activate<kMode>(gate, up, a.limit, a.alpha));
                            } else {
                                const int r0 = tile * 16 + g;
                                float* y = a.w.ybuf + (int64_t)sl * a.H;
                                y[r0] = (y0 + bias0[ti]) * mul;
                                y[r0 + 8] = (y1 + bias1[ti]) * mul;
                            }
                        }
                    }
                }
            }
        }
    }
    __syncthreads();
    // the last CTA to finish resets the work counters for the next launch
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(&a.w.sched[1], 1u) == gridDim.x - 1) {
            a.w.sched[0] = 0;
            a.w.sched[1] = 0;
            __threadfence();
        }
    }
}

// K-split (1, 2 or 4 warps per tile): the smallest that gives the launch
// about one work item per SM (measured best at batch 1: a second round of
// items on an SM costs more than the split's reduction), keeping at least
// two 8-block groups per split.
int pick_split(int experts, int ntiles, int ngrp) {
    int ks = 1;
    while (ks < 4 && ks * 2 <= std::max(1, ngrp / 2) && (int64_t)experts * ((ntiles * ks + kCT - 1) / kCT) < 118)
        ks *= 2;
    return ks;
}

}  // namespace

int configure_expert_gemv() {
    const int bytes = smem_plan(kMaxGemvCols).total;
    for (auto fn : {k_expert_gemv<0>, k_expert_gemv<1>, k_expert_gemv<2>})
        if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) return -1;
    return 0;
}

bool expert_gemv_supported(const MoeDims& d) {
    return d.H <= kMaxGemvCols && d.F <= kMaxGemvCols && tensor_map_encoder() != nullptr;
}

int launch_expert_gemv(const LayerView& L, const MoeDims& d, const MoeWork& w, int T, int which,
                       cudaStream_t s) {
    ExpertGemvArgs a;
    a.base = L.base;
    a.stride = L.stride;
    int64_t off_pk, off_sc;
    if (which == 0) {
        a.M = 2 * d.F; a.K = d.H;
        off_pk = L.off[0]; off_sc = L.off[1]; a.off_bias = L.off[4];
    } else {
        a.M = d.H; a.K = d.F;
        off_pk = L.off[2]; off_sc = L.off[3]; a.off_bias = L.off[5];
    }
    if (a.K > kMaxGemvCols || a.K % 32 || a.M % 16) return -1;
    a.k = d.k;
    a.shard_count = d.shard_count;
    a.F = d.F;
    a.H = d.H;
    a.limit = d.limit;
    a.alpha = d.alpha;
    a.w = w;
    const int nblk = a.K / 32, nfull = nblk / 8, ntiles = a.M / 16;
    const int wlast = nblk - 8 * ((nblk + 7) / 8 - 1);
    const int e_local = (d.E - d.shard_rank + d.shard_count - 1) / d.shard_count;
    const int maxa = std::min(d.E, T * d.k);
    a.ksplit = pick_split(maxa, ntiles, (nblk + 7) / 8);
    const int tb = kCT / a.ksplit;
    // TMA views of the bank (uint8 elements; a tile is 16 * nblk * 16 bytes
    // of blocks and 16 * nblk bytes of scales; experts one stride apart):
    //   w_full   (128 B, 16 rows, full groups, tiles, experts), box (128, 16, 1, tb, 1), 128-byte swizzle
    //   w_narrow (16 w B, 16 rows, tiles, experts) at the last group, box (16 w, 16, tb, 1)
    //   s_full   (128 B, full groups, tiles, experts), box (128, 1, tb, 1)
    //   s_narrow (16 w B, tiles, experts) at the last group, box (16 w, tb, 1)
    // A view whose groups do not exist (no full or no narrow group) is encoded
    // over the first group and never used.
    GemvMaps maps;
    auto enc = tensor_map_encoder();
    if (!enc) return -1;
    const uint8_t* pk = L.base + off_pk;
    const uint8_t* sc = L.base + off_sc;
    const cuuint64_t tile_pk = (cuuint64_t)nblk * 256, tile_sc = (cuuint64_t)nblk * 16, es = (cuuint64_t)L.stride;
    const int wn = wlast < 8 ? wlast : 8;
    const cuuint64_t nf = nfull > 0 ? nfull : 1;
    const cuuint32_t ones[5] = {1, 1, 1, 1, 1};
    bool good = true;
    {
        const cuuint64_t gd[5] = {128, 16, nf, (cuuint64_t)ntiles, (cuuint64_t)e_local};
        const cuuint64_t gs[4] = {128, 2048, tile_pk, es};
        const cuuint32_t box[5] = {128, 16, 1, (cuuint32_t)kBoxT, 1};
        good = good && enc(&maps.w_full, CU_TENSOR_MAP_DATA_TYPE_UINT8, 5, const_cast<uint8_t*>(pk), gd, gs, box,
                           ones, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    }
    {
        const cuuint64_t gd[4] = {(cuuint64_t)16 * wn, 16, (cuuint64_t)ntiles, (cuuint64_t)e_local};
        const cuuint64_t gs[3] = {(cuuint64_t)16 * wn, tile_pk, es};
        const cuuint32_t box[4] = {(cuuint32_t)(16 * wn), 16, (cuuint32_t)kBoxT, 1};
        good = good && enc(&maps.w_narrow, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4,
                           const_cast<uint8_t*>(pk + (wlast < 8 ? (int64_t)nfull * 2048 : 0)), gd, gs, box, ones,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    }
    {
        const cuuint64_t gd[4] = {128, nf, (cuuint64_t)ntiles, (cuuint64_t)e_local};
        const cuuint64_t gs[3] = {128, tile_sc, es};
        const cuuint32_t box[4] = {128, 1, (cuuint32_t)tb, 1};
        good = good && enc(&maps.s_full, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<uint8_t*>(sc), gd, gs, box,
                           ones, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    }
    {
        const cuuint64_t gd[3] = {(cuuint64_t)16 * wn, (cuuint64_t)ntiles, (cuuint64_t)e_local};
        const cuuint64_t gs[2] = {tile_sc, es};
        const cuuint32_t box[3] = {(cuuint32_t)(16 * wn), (cuuint32_t)tb, 1};
        good = good && enc(&maps.s_narrow, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3,
                           const_cast<uint8_t*>(sc + (wlast < 8 ? (int64_t)nfull * 128 : 0)), gd, gs, box, ones,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    }
    if (!good) return -1;
    // persistent: one CTA per SM, or one per work item when there are fewer
    static int sms[16] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 16) return -1;
    if (!sms[dev] && cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return -1;
    const int items = (maxa + T * d.k / kEPass) * ((ntiles + tb - 1) / tb);
    const dim3 grid(std::min(items, sms[dev]));
    const int smem = smem_plan(a.K).total;
    if (which == 1) k_expert_gemv<2><<<grid, kEThreads, smem, s>>>(maps, a);
    else if (d.act == 0) k_expert_gemv<0><<<grid, kEThreads, smem, s>>>(maps, a);
    else k_expert_gemv<1><<<grid, kEThreads, smem, s>>>(maps, a);
    return cudaPeekAtLastError() == cudaSuccess ? 1 : -1;
}

}  // namespace gw
