// gw_grouped.cu — the prefill expert GEMMs on the 5th-generation tensor cores.
//
// When many tokens share an expert (prefill, large batches) the expert FFN is
// a grouped GEMM: for each active expert e, D_e[rows][tokens] = W_e x_e^T with
// W_e the expert's MXFP4 matrix (gate_up: 2F x H, down: H x F) and x_e the
// rows of the tokens routed to it.  The reference applies each (expert, token)
// assignment separately as mxfp4_gemv_bias -> activation -> mxfp4_gemv_bias
// -> expert_accumulate (ExpertRunner.applyAssignments,
// Runtime/ExpertRunner.swift:108-183); this kernel computes the same values —
// fp32 sums of f16 activations times MXFP4 weights, bias, clamped SwiGLU into
// f16, down projection times the routing weight — for all of an expert's
// tokens from one pass over its weights.
//
// Two kernels share the work list and the epilogue: k_grouped (exact f16
// operands, described here) and k_grouped_mx (block-scaled MXFP4 x MXFP8,
// described above its roles further down).
//
// One persistent CTA per SM walks a static list of work items (128-row tile,
// expert, token chunk of <= 128).  Warp roles of k_grouped:
//   warp 12     weight producer: bulk-copies (cp.async.bulk) each 8-block
//               group of the tile — in the bank's tiled layout a contiguous
//               16 x w x 16-byte run per 16-row tile, plus its scale bytes —
//               into a 3-group shared ring (mbarrier transaction counts
//               signal arrival).
//   warps 0-7   converters: widen each stage (128 rows x up to 128 columns)
//               to f16 (cvt.rn.f16x2.e2m1x2, times the block scale) straight
//               into tensor memory (tcgen05.st: thread = row = TMEM lane), a
//               4-stage ring of 64 columns each.
//   warp 13     token producer: one or two 2D TMAs (128 rows x 64 columns,
//               128B swizzle) per stage from the expert-ordered f16 token rows
//               (x16 gathered by k_gather for gate_up; the gate_up epilogue
//               writes its activations in that order for down) into a 4-stage
//               shared ring.
//   warp 14     MMA issuer: one lane, tcgen05.mma kind::f16 M=128 N=n K=16
//               with A in TMEM and B in shared memory, fp32 accumulators in
//               TMEM (two 128-column buffers so the epilogue of one item
//               overlaps the main loop of the next).
//   warps 8-11  epilogue: tcgen05.ld the accumulators (one row per thread),
//               scale, bias, activation / routing weight, store.
// Every wait is bounded (~2 s); a wait that runs out sets a bit in the
// workspace status word and makes the whole CTA wind down: it lets its copies
// land, waits for its MMAs and frees its TMEM before returning.
//
// f16 operands are exact: x16 rows are the router's power-of-two-shifted
// activations, and each weight row is multiplied by 2^(128 - emax_row) with
// emax_row the row's largest biased E8M0 exponent (precomputed per bank row):
// the row's largest blocks then hold e2m1 x 2^1 (at most 12) and every block
// within 25 binades of them is exact in f16 (normal or subnormal); blocks
// further down, whose products are below 2^-25 of the row's largest, flush to
// zero.  The epilogue undoes both shifts in fp32.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <mutex>
#include <type_traits>

#include "gw_async.cuh"
#include "gw_device.cuh"
#include "gw_internal.h"

namespace gw {
namespace {

constexpr int kM = 128;                   // weight rows per tile (MMA M)
constexpr int kNMax = 128;                // token columns per chunk (MMA N max)
constexpr int kKS = 128;                  // columns per stage (up to four MXFP4 blocks)
constexpr int kStages = 4;                // operand ring the MMA reads
constexpr int kGroups = 3;                // raw weight ring, in 8-block groups
constexpr int kBox = 64;                  // token columns per TMA box (one 128-byte swizzled row)
constexpr int kBBox = kNMax * kBox * 2;   // 16 KB: one box of token rows
constexpr int kBSlot = 2 * kBBox;         // 32 KB of f16 tokens per stage
constexpr int kACols = kKS / 2;           // TMEM columns of one stage's f16 weights (2 per column)
constexpr int kTileRun = 16 * 8 * 16;     // one 16-row tile's blocks of a full group
constexpr int kGroupPk = 8 * kTileRun;    // 16 KB of MXFP4 blocks per group
constexpr int kGroupSc = 8 * 16 * 8;      // 1 KB of scale bytes per group
constexpr int kRingBytes = kStages * kBSlot;
constexpr int kGroupOff = kRingBytes;
constexpr int kDynSmem = kGroupOff + kGroups * (kGroupPk + kGroupSc) + 1024;  // + alignment slack
constexpr int kThreads = 15 * 32;
constexpr int kTmemCols = 512;            // accumulators 2 x kNMax, then the weight ring
constexpr int kAColBase = 2 * kNMax;
static_assert(kAColBase + kStages * kACols <= kTmemCols, "TMEM budget");

// Warp roles.
constexpr int kConvWarps = 8, kEpiWarp0 = 8, kWeightWarp = 12, kTokenWarp = 13, kMmaWarp = 14;

struct GroupedArgs {
    LayerView L;
    MoeDims d;
    MoeWork w;
    int M, K;                 // rows and columns of the expert matrix
    int sec_packed, sec_scales, sec_bias;
    int rexp_off;             // row offset of this matrix in the row-exponent table
    int bdiv;                 // token row = slot / bdiv
    int mode;                 // 0 gate_up clamped GLU, 1 gate_up SiLU, 2 down
    const uint32_t* bsf;      // block-scaled mode: token scale words [rows][ceil(K/128)]
};

// ---- PTX wrappers (the mbarrier / bulk-copy ones are in gw_async.cuh) ------
// One 2D tile of `map` at (x, y) -> shared, counted on `b`.
__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* b) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
        "%3}], [%4];" ::"r"(saddr(dst)),
        "l"(map), "r"(x), "r"(y), "r"(saddr(b))
        : "memory");
}
__device__ __forceinline__ void tc_after_sync() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_before_sync() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* b) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     saddr(b))
                 : "memory");
}
// The same with A read from tensor memory (128 lanes = rows, two f16 per
// 32-bit column along K).
__device__ __forceinline__ void tc_mma_ta(uint32_t tmem, uint32_t a_tmem, uint64_t bd, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem),
        "r"(a_tmem), "l"(bd), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Block-scaled MMA: A e2m1 and B e4m3 from shared memory (descriptors), fp32
// accumulators in TMEM, E8M0 scale factors in TMEM at sfa / sfb (the byte
// used is chosen by the instruction descriptor's scale-factor ids).
__device__ __forceinline__ void tc_mma_mx(uint32_t tmem, uint64_t ad, uint64_t bd, uint32_t idesc,
                                          uint32_t accumulate, uint32_t sfa, uint32_t sfb) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(tmem),
        "l"(ad), "l"(bd), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
        : "memory");
}
// Shared -> TMEM copies of the block-scaled mode's scale words, issued by the
// MMA thread ahead of the stage's MMAs (the tensor pipe keeps them in order):
// 128 rows x 16 bytes to lanes 0-127, and 32 rows x 16 bytes to lanes 0-31 of
// every lane quarter.
__device__ __forceinline__ void tc_cp_128x128b(uint32_t taddr, uint64_t sdesc) {
    asm volatile("tcgen05.cp.cta_group::1.128x128b [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}
__device__ __forceinline__ void tc_cp_32x128b_x4(uint32_t taddr, uint64_t sdesc) {
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}
// 32 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
        "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
        "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// Shared-memory matrix descriptor, K-major.  layout 0 = no swizzle (core
// matrices of 8 rows x 16 bytes; lbo = distance between the two K-adjacent
// core matrices of one MMA, sbo = distance between 8-row groups); layout 2 =
// 128-byte swizzle (rows of 128 bytes, sbo = 1024 between 8-row atoms).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | ((uint64_t)1 << 46) | ((uint64_t)layout << 61);
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// e2m1 pair (one packed byte) -> f16x2, low nibble in the low half.
__device__ __forceinline__ uint32_t e2m1x2(uint32_t byte) {
    uint32_t h2;
    asm("{\n\t.reg .b8 q;\n\tcvt.u8.u32 q, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, q;\n\t}" : "=r"(h2) : "r"(byte));
    return h2;
}

// f16x2 bit pattern of 2^(sb - emax + 1) (both halves), the factor that
// takes e2m1x2's output to e2m1 * 2^(sb - emax + 1): 0 for scale byte 0
// and below f16's smallest subnormal, +inf for scale byte 255 (the fp32 GEMV
// path's 2^(sb-127) bit pattern gives 0 and inf for those bytes too).
__device__ __forceinline__ uint32_t block_scale_h2(uint32_t sb, int emax) {
    uint32_t h;
    if (sb == 0) h = 0;
    else if (sb == 255) h = 0x7C00u;
    else {
        const int p = (int)sb - emax + 1;
        if (p >= -14) h = (uint32_t)(p + 15) << 10;
        else if (p >= -24) h = 1u << (p + 24);
        else h = 0;
    }
    return h | (h << 16);
}

__device__ __forceinline__ uint32_t hmul2_bits(uint32_t a, uint32_t b) {
    __half2 r = __hmul2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
}

struct Shared {
    uint64_t full[kStages], empty[kStages], gfull[kGroups], gempty[kGroups], tfull[2], tempty[2], fin;
    uint32_t tmem;
    int abort;
    int nact, nitems, chunks, mt;
    int prefix[kMaxExperts + 1];  // token chunks before active expert a
    int expert[kMaxExperts];
    int count[kMaxExperts];
    int goff[kMaxExperts];        // first expert-ordered row of active expert a
    int epre[kMaxExperts];        // expert-ordered rows before expert e (all experts)
    int col_slot[kNMax];          // epilogue: slot of each token column
    float col_mul[kNMax];         // epilogue: xmul (gate_up) or routing weight (down)
};

struct Item {
    int e, m0, c0, n;
    int g0;  // expert-ordered row of the chunk's first token
};

// Items are numbered chunk-major (item = j * mt + m): the row tiles of one
// token chunk run at about the same time on neighbouring CTAs, so the chunk's
// token rows come from DRAM once and from L2 for the other tiles.
__device__ __forceinline__ Item decode(const Shared& sh, int it) {
    const int j = it / sh.mt, m = it - j * sh.mt;
    Item r;
    r.m0 = m * kM;
    int lo = 0, hi = sh.nact;
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (sh.prefix[mid] <= j) lo = mid; else hi = mid;
    }
    r.e = sh.expert[lo];
    r.c0 = (j - sh.prefix[lo]) * kNMax;
    r.n = min(kNMax, sh.count[lo] - r.c0);
    r.g0 = sh.goff[lo] + r.c0;
    return r;
}

// ---- roles ----------------------------------------------------------------
//
// A K-range of an item is walked in stages of up to four 32-column blocks
// that never straddle an 8-block group: a group of w blocks (w = 8, or the
// even remainder of the last group) is ceil(w / 4) stages of 4, 4 or 2 blocks.

// Weight producer (one warp, converged): for every item, every 8-block group
// of its 128-row tile, once the ring slot is free; lane t copies tile t.
__device__ __forceinline__ void role_weights(Shared& sh, const GroupedArgs& a, char* smem) {
    const int nblk = a.K >> 5, ngrp = (nblk + 7) >> 3;
    const int lane = threadIdx.x & 31;
    unsigned* status = a.w.status;
    char* ring = smem + kGroupOff;
    int gq = 0;
    for (int it = blockIdx.x; it < sh.nitems; it += gridDim.x) {
        const Item item = decode(sh, it);
        const int64_t le = item.e / a.d.shard_count;
        const uint8_t* ex = a.L.base + le * a.L.stride;
        const int64_t tile0 = item.m0 >> 4;
        const uint8_t* pk = ex + a.L.off[a.sec_packed] + tile0 * 16 * nblk * 16;
        const uint8_t* sc = ex + a.L.off[a.sec_scales] + tile0 * 16 * nblk;
        const int tiles = min(8, (a.M - item.m0) >> 4);
        for (int grp = 0; grp < ngrp; ++grp, ++gq) {
            const int slot = gq % kGroups;
            if (!warp_wait(&sh.abort, &sh.gempty[slot], ((gq / kGroups) & 1) ^ 1, status, 1u)) return;
            const int w = min(8, nblk - 8 * grp);
            const uint32_t run = 16 * w * 16, srun = 16 * w;  // bytes per tile: blocks, scales
            char* dpk = ring + slot * (kGroupPk + kGroupSc);
            char* dsc = dpk + kGroupPk;
            if (lane == 0) bar_arrive_tx(&sh.gfull[slot], tiles * (run + srun));
            __syncwarp();
            if (lane < tiles) {
                const int t = lane;
                bulk_g2s(dpk + t * kTileRun, pk + (int64_t)t * 16 * nblk * 16 + grp * 128 * 16, run,
                         &sh.gfull[slot]);
                bulk_g2s(dsc + t * 128, sc + (int64_t)t * 16 * nblk + grp * 128, srun, &sh.gfull[slot]);
            }
        }
    }
}

// Converters: thread c owns weight row m0 + (c & 127) — its TMEM lane — and,
// of each stage's up-to-four blocks, blocks 2h and 2h + 1 (h = c >> 7),
// which it widens to 64 f16 and stores as 32 TMEM columns.  Lane 0 of each
// warp does the barrier work for its warp.
__device__ __forceinline__ void role_convert(Shared& sh, const GroupedArgs& a, char* smem) {
    const int c = threadIdx.x;
    const int r = c & (kM - 1), h = c >> 7, lane = c & 31, warp = c >> 5;
    const int lr = r & 15, tile = r >> 4;
    const int nblk = a.K >> 5, ngrp = (nblk + 7) >> 3;
    unsigned* status = a.w.status;
    const char* ring = smem + kGroupOff;
    const uint32_t tlane = (uint32_t)((warp & 3) * 32) << 16;
    auto row_emax = [&](int it) -> int {
        if (it >= sh.nitems) return 127;
        const Item item = decode(sh, it);
        const int R = item.m0 + r;
        if (R >= a.M) return 127;
        return a.L.rowexp[(int64_t)(item.e / a.d.shard_count) * a.L.rowexp_stride + a.rexp_off + R];
    };
    int emax_next = row_emax(blockIdx.x);
    int g = 0, gq = 0;
    bool ok = true;
    for (int it = blockIdx.x; ok && it < sh.nitems; it += gridDim.x) {
        const Item item = decode(sh, it);
        const bool valid = item.m0 + r < a.M;
        const int emax = emax_next;
        emax_next = row_emax(it + gridDim.x);  // lands while this item runs
        for (int grp = 0; ok && grp < ngrp; ++grp, ++gq) {
            const int w = min(8, nblk - 8 * grp);
            const int gslot = gq % kGroups;
            if (!warp_wait(&sh.abort, &sh.gfull[gslot], (gq / kGroups) & 1, status, 2u)) { ok = false; break; }
            const char* gb = ring + gslot * (kGroupPk + kGroupSc);
            for (int sub = 0; sub * 4 < w; ++sub, ++g) {
                const int kb = min(4, w - 4 * sub);  // blocks in this stage (4 or 2)
                const bool mine = 2 * h < kb;        // this thread's two blocks exist
                const int bl = 4 * sub + 2 * h;      // its first block within the group
                uint32_t v[32];
                if (valid && mine) {
                    const uint4* q = reinterpret_cast<const uint4*>(gb + tile * kTileRun + (lr * w + bl) * 16);
                    const uint8_t* sb = reinterpret_cast<const uint8_t*>(gb + kGroupPk + tile * 128 + lr * w + bl);
#pragma unroll
                    for (int b2 = 0; b2 < 2; ++b2) {
                        const uint4 qq = q[b2];
                        const uint32_t hs = block_scale_h2(sb[b2], emax);
                        const uint32_t wd[4] = {qq.x, qq.y, qq.z, qq.w};
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            v[16 * b2 + 4 * j + 0] = hmul2_bits(e2m1x2(wd[j] & 0xFF), hs);
                            v[16 * b2 + 4 * j + 1] = hmul2_bits(e2m1x2((wd[j] >> 8) & 0xFF), hs);
                            v[16 * b2 + 4 * j + 2] = hmul2_bits(e2m1x2((wd[j] >> 16) & 0xFF), hs);
                            v[16 * b2 + 4 * j + 3] = hmul2_bits(e2m1x2(wd[j] >> 24), hs);
                        }
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = 0;
                }
                if (4 * sub + 4 >= w) {  // the group's last stage has been read: free its slot
                    __syncwarp();
                    if (lane == 0) bar_arrive(&sh.gempty[gslot]);
                }
                const int slot = g % kStages;
                if (!warp_wait(&sh.abort, &sh.empty[slot], ((g / kStages) & 1) ^ 1, status, 4u)) { ok = false; break; }
                // the warp's 32 rows, columns [32h, 32h + 32) of the stage's weight slot
                if (2 * h < kb) {  // uniform over the warp
                    tmem_st32(sh.tmem + tlane + kAColBase + slot * kACols + 32 * h, v);
                    tmem_st_wait();
                }
                tc_before_sync();
                __syncwarp();
                if (lane == 0) bar_arrive(&sh.full[slot]);
            }
        }
    }
}

// Token producer (one warp, converged; lane 0 issues): the chunk's rows are
// consecutive in the expert-ordered token matrix, so each stage is one or two
// 2D TMAs of 128 rows x 64 columns (rows past the chunk belong to the next
// expert and only fill columns the epilogue ignores; rows past the matrix
// read as zero).
__device__ __forceinline__ void role_tokens(Shared& sh, const GroupedArgs& a, char* smem,
                                            const CUtensorMap* map) {
    const int nblk = a.K >> 5, ngrp = (nblk + 7) >> 3;
    const int lane = threadIdx.x & 31;
    unsigned* status = a.w.status;
    int g = 0;
    for (int it = blockIdx.x; it < sh.nitems; it += gridDim.x) {
        const Item item = decode(sh, it);
        for (int grp = 0; grp < ngrp; ++grp) {
            const int w = min(8, nblk - 8 * grp);
            for (int sub = 0; sub * 4 < w; ++sub, ++g) {
                const int kb = min(4, w - 4 * sub);
                const int slot = g % kStages;
                if (!warp_wait(&sh.abort, &sh.empty[slot], ((g / kStages) & 1) ^ 1, status, 8u)) return;
                if (lane == 0) {
                    char* B = smem + slot * kBSlot;
                    const int x0 = (8 * grp + 4 * sub) * 32;
                    bar_arrive_tx(&sh.full[slot], (uint32_t)(kb / 2) * kBBox);
                    for (int cb = 0; cb < kb / 2; ++cb)
                        tma_2d(B + cb * kBBox, map, x0 + cb * kBox, item.g0, &sh.full[slot]);
                }
                __syncwarp();
            }
        }
    }
}

// MMA issuer: one warp, converged; lane 0 issues.  A stage of kb blocks is
// 2 kb MMAs of K = 16: A from the stage's TMEM columns, B from its shared
// slot (box cb = k / 4, 32 bytes per K step inside the swizzled row).
__device__ __forceinline__ void role_mma(Shared& sh, const GroupedArgs& a, char* smem) {
    const int nblk = a.K >> 5, ngrp = (nblk + 7) >> 3;
    const int lane = threadIdx.x & 31;
    unsigned* status = a.w.status;
    const uint32_t base = saddr(smem);
    int g = 0, il = 0;
    bool ok = true;
    for (int it = blockIdx.x; ok && it < sh.nitems; it += gridDim.x, ++il) {
        const Item item = decode(sh, it);
        const int n = max(16, (item.n + 15) & ~15);
        const uint32_t idesc = (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kM >> 4) << 24);
        const int b = il & 1;
        if (!warp_wait(&sh.abort, &sh.tempty[b], ((il >> 1) & 1) ^ 1, status, 16u)) break;
        tc_after_sync();
        const uint32_t dtm = sh.tmem + b * kNMax;
        bool first = true;
        for (int grp = 0; ok && grp < ngrp; ++grp) {
            const int w = min(8, nblk - 8 * grp);
            for (int sub = 0; sub * 4 < w; ++sub, ++g) {
                const int kb = min(4, w - 4 * sub);
                const int slot = g % kStages;
                if (!warp_wait(&sh.abort, &sh.full[slot], (g / kStages) & 1, status, 32u)) { ok = false; break; }
                tc_after_sync();
                if (lane == 0) {
                    const uint32_t atm = sh.tmem + kAColBase + slot * kACols;
                    const uint32_t B = base + slot * kBSlot;
                    for (int k = 0; k < 2 * kb; ++k) {
                        tc_mma_ta(dtm, atm + k * 8, smem_desc(B + (k >> 2) * kBBox + (k & 3) * 32, 16, 1024, 2),
                                  idesc, first ? 0u : 1u);
                        first = false;
                    }
                    tc_commit(&sh.empty[slot]);
                }
                __syncwarp();
            }
        }
        if (!ok) break;
        if (lane == 0) tc_commit(&sh.tfull[b]);
        __syncwarp();
    }
    // every MMA this warp issued has finished before TMEM is freed
    if (lane == 0) {
        tc_commit(&sh.fin);
        const long long t0 = clock64();
        while (!bar_try(&sh.fin, 0)) {
            if (clock64() - t0 > kWaitCycles) {
                if (status) atomicOr(status, 64u);
                break;
            }
        }
    }
    __syncwarp();
}

// ---- block-scaled roles (gw_set_block_scaled) ------------------------------




// Epilogue: thread t (0..127) owns TMEM lane t = tile row m0 + t.
template <int kMode, bool kMX>
__device__ __forceinline__ void role_epilogue(Shared& sh, const GroupedArgs& a) {
    const int t = threadIdx.x - kEpiWarp0 * 32;
    const int ew = t >> 5, lane = t & 31;
    unsigned* status = a.w.status;
    int il = 0;
    for (int it = blockIdx.x; it < sh.nitems; it += gridDim.x, ++il) {
        const Item item = decode(sh, it);
        const int R = item.m0 + t;
        const bool valid = R < a.M;
        const int64_t le = item.e / a.d.shard_count;
        const uint8_t* ex = a.L.base + le * a.L.stride;
        const uint16_t* bias = reinterpret_cast<const uint16_t*>(ex + a.L.off[a.sec_bias]);
        // the f16 path's weights carry the row shift 2^(1 - emax); the block-scaled
        // path's products are already in the true scale
        const int emax = kMX ? 128 : (valid ? (int)a.L.rowexp[le * a.L.rowexp_stride + a.rexp_off + R] : 127);
        const float bv = valid ? bf16_bits_to_f32(bias[R]) : 0.f;
        const int p = emax - 128, p1 = p / 2;  // undoes the 2^(1 - emax) row shift
        const float rs1 = pow2f(p1), rs2 = pow2f(p - p1);
        // column metadata for the chunk, one column per thread
        const int32_t* list = a.w.lists + (int64_t)item.e * a.w.tcap + item.c0;
        static_assert(kNMax == 128, "one column per epilogue thread");
        const int cs = t < item.n ? __ldg(list + t) : 0;
        const float cm = t < item.n ? (kMode == 2 ? a.w.weights[cs] : (kMX ? 1.f : a.w.xmul[cs / a.d.k])) : 0.f;
        group_sync(1, 128);
        sh.col_slot[t] = cs;
        sh.col_mul[t] = cm;
        group_sync(1, 128);
        const int b = il & 1;
        const bool got = wait_on(&sh.abort, &sh.tfull[b], (il >> 1) & 1, status, 128u);
        if (group_any(!got, 2, 128)) break;
        tc_after_sync();
        const uint32_t taddr = sh.tmem + b * kNMax + ((uint32_t)(ew * 32) << 16);
        const float pbv = __shfl_xor_sync(0xffffffffu, bv, 1);
        for (int j0 = 0; j0 < item.n; j0 += 16) {
            float v[16];
            tmem_ld16(taddr + j0, v);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int col = j0 + j;
                const float acc = v[j] * rs1 * rs2;
                if (kMode == 2) {
                    if (valid && col < item.n)
                        a.w.ybuf[(int64_t)sh.col_slot[col] * a.M + R] = (acc + bv) * sh.col_mul[col];
                } else {
                    const float partner = __shfl_xor_sync(0xffffffffu, acc, 1);
                    if (valid && (lane & 1) == 0 && col < item.n) {
                        const float xm = sh.col_mul[col];
                        const float y = activate<kMode>(acc * xm + bv, partner * xm + pbv, a.d.limit, a.d.alpha);
                        a.w.act[(int64_t)(item.g0 + col) * a.d.F + (R >> 1)] = __float2half_rn(y);
                    }
                }
            }
        }
        tc_before_sync();
        bar_arrive(&sh.tempty[b]);
    }
}

// Work list of a launch (every CTA computes the same): the active experts,
// their token-chunk prefix, and the expert-ordered row offsets.
__device__ __forceinline__ void plan_items(Shared& sh, const GroupedArgs& a) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int mt = (a.M + kM - 1) / kM;
    // active experts and their token chunks
    const int nact = min(*a.w.nactive, a.d.E);
    for (int i = tid; i < nact; i += blockDim.x) {
        const int e = a.w.active[i];
        const int cnt = min(a.w.counts[e], a.w.tcap);
        sh.expert[i] = e;
        sh.count[i] = cnt;
        sh.prefix[i + 1] = (cnt + kNMax - 1) / kNMax;
    }
    if (tid == 0) {
        sh.abort = 0;
        sh.nact = nact;
    }
    __syncthreads();
    if (warp == 0) {  // exclusive prefix over <= 256 chunk counts, 8 per lane
        int v[8], sum = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int i = lane * 8 + j;
            v[j] = i < nact ? sh.prefix[i + 1] : 0;
            sum += v[j];
        }
        int incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        int run = incl - sum;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int i = lane * 8 + j;
            if (i < nact) sh.prefix[i] = run;
            run += v[j];
        }
        if (lane == 31) { sh.prefix[nact] = incl; sh.chunks = incl; sh.mt = mt; sh.nitems = incl * mt; }
    } else if (warp == 1) {  // expert-ordered row offsets: exclusive prefix over all experts' counts
        int v[8], sum = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int e = lane * 8 + j;
            v[j] = e < a.d.E ? min(a.w.counts[e], a.w.tcap) : 0;
            sum += v[j];
        }
        int incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        int run = incl - sum;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int e = lane * 8 + j;
            if (e < a.d.E) sh.epre[e] = run;
            run += v[j];
        }
    }
    __syncthreads();
    for (int i = tid; i < nact; i += blockDim.x) sh.goff[i] = sh.epre[sh.expert[i]];
    __syncthreads();
}

// ---- block-scaled mode: weights by TMA straight into the MMA's layout -------
//
// k_grouped_mx: the block-scaled grouped GEMM with one stage per 8-block group
// (K = 256, eight MMAs) and no conversion role.  Per stage:
//   warp 12 (lane 0)  weights: two TMA boxes of the bank's tiled layout viewed
//                     as 4-bit elements (CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B),
//                     128 rows x 128 values each, which the copy unpacks into
//                     the MMA's e2m1 layout (16 values in 8 bytes + 8 bytes of
//                     padding) with the 128-byte swizzle; tokens: two boxes of
//                     128 E4M3 codes x 128 rows; one transaction count.
//   warp 13           scale words: the tile rows' E8M0 bytes of the group and
//                     the tokens' words, staged for tcgen05.cp.
//   warp 14 (lane 0)  tcgen05.cp of both scale sets into TMEM, then eight
//                     kind::mxf8f6f4.block_scale MMAs (M = 128, K = 32) from
//                     the 128-byte-swizzled operands, one commit.
//   warps 8-11        epilogue (as the f16 path's).
// The last group of a row (w < 8 blocks) is a stage of w MMAs from boxes of
// a 4-D view whose rows are 16 w bytes apart; the box's values beyond the
// row read as zeros and are not used.
constexpr int kS2 = 3;                        // stages in flight
constexpr int kS2A = kM * 256 / 2 * 2;        // 32 KB: 128 rows x 256 unpacked e2m1 (1 byte / value)
constexpr int kS2B = kNMax * 256;             // 32 KB: 128 tokens x 256 E4M3 codes
constexpr int kS2Sa = 2 * kM * 16;            // 4 KB: two 128 x 16-byte scale-word slabs
constexpr int kS2Sb = 2 * 32 * 16;            // 1 KB: two 32 x 16-byte token-word slabs
constexpr int kS2Slot = kS2A + kS2B + kS2Sa + kS2Sb;
constexpr int kS2Smem = kS2 * kS2Slot + 1024;
constexpr int kS2Sfa = 2 * kNMax;             // TMEM columns: weight scale words, 8 per stage
constexpr int kS2Sfb = kS2Sfa + 8 * kS2;      // token scale words, 8 per stage
static_assert(kS2Sfb + 8 * kS2 <= kTmemCols, "TMEM budget");
static_assert(kS2 <= kStages, "barrier arrays");

struct MxMaps {
    CUtensorMap b;        // token codes [rows][K], box 128 codes x 32 rows, 128-byte swizzle
    CUtensorMap wfull;    // 16U4 (256 values, 16 rows, full groups, tiles, experts), box (128, 16, 1, 8, 1)
    CUtensorMap wnarrow;  // 16U4 (32 w values, 16 rows, tiles, experts) at the last group, box (128, 16, 8, 1)
};

__device__ __forceinline__ void tma_4d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                       uint64_t* b) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
        "%4, %5}], [%6];" ::"r"(saddr(dst)),
        "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(saddr(b))
        : "memory");
}
__device__ __forceinline__ void tma_5d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3, int c4,
                                       uint64_t* b) {
    asm volatile(
        "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
        "%4, %5, %6}], [%7];" ::"r"(saddr(dst)),
        "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(saddr(b))
        : "memory");
}

// Weight and token copies (lane 0 of warp 12).
__device__ __forceinline__ void role_copies_mx2(Shared& sh, const GroupedArgs& a, char* smem, const MxMaps* maps) {
    const int nblk = a.K >> 5, ngrp = (nblk + 7) >> 3, nfull = nblk >> 3;
    unsigned* status = a.w.status;
    int g = 0;
    for (int it = blockIdx.x; it < sh.nitems; it += gridDim.x) {
        const Item item = decode(sh, it);
        const int le = item.e / a.d.shard_count;
        const int tile0 = item.m0 >> 4;
        for (int grp = 0; grp < ngrp; ++grp, ++g) {
            const int slot = g % kS2;
            if (!wait_on(&sh.abort, &sh.empty[slot], ((g / kS2) & 1) ^ 1, status, 1u)) return;
            const int w = min(8, nblk - 8 * grp);
            const int nbox = (w + 3) >> 2;          // 128-value boxes
            const int nrow = (item.n + 31) >> 5;    // 32-token boxes: only the chunk's rows
            char* A = smem + slot * kS2Slot;
            char* B = A + kS2A;
            // packed weight bytes (the transaction counts the global bytes,
            // 64 per row and box) plus the token codes
            bar_arrive_tx(&sh.full[slot], (uint32_t)nbox * (kM * 64 + nrow * 32 * 128));
            for (int x = 0; x < nbox; ++x) {
                if (grp < nfull) tma_5d(A + x * (kS2A / 2), &maps->wfull, 128 * x, 0, grp, tile0, le, &sh.full[slot]);
                else tma_4d(A + x * (kS2A / 2), &maps->wnarrow, 128 * x, 0, tile0, le, &sh.full[slot]);
                for (int y = 0; y < nrow; ++y)
                    tma_2d(B + x * (kS2B / 2) + y * 32 * 128, &maps->b, grp * 256 + 128 * x, item.g0 + 32 * y,
                           &sh.full[slot]);
            }
        }
    }
}

// Scale words (warp 13): lane l stages rows 4l .. 4l + 3 of the tile and the
// tokens l, 32 + l, 64 + l, 96 + l.
__device__ __forceinline__ void role_scales_mx2(Shared& sh, const GroupedArgs& a, char* smem) {
    const int nblk = a.K >> 5, ngrp = (nblk + 7) >> 3, nst = (a.K + 127) >> 7;
    const int lane = threadIdx.x & 31;
    unsigned* status = a.w.status;
    int g = 0;
    for (int it = blockIdx.x; it < sh.nitems; it += gridDim.x) {
        const Item item = decode(sh, it);
        const int64_t le = item.e / a.d.shard_count;
        const uint8_t* sc = a.L.base + le * a.L.stride + a.L.off[a.sec_scales];
        for (int grp = 0; grp < ngrp; ++grp, ++g) {
            const int slot = g % kS2;
            const int w = min(8, nblk - 8 * grp);
            // the rows' scale bytes: in the tiled layout tile t's group holds
            // 16 rows x w bytes from t * 16 * nblk + grp * 128
            uint32_t rw[4][2];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int r = 4 * lane + q, R = item.m0 + r;
                rw[q][0] = rw[q][1] = 0u;
                if (R < a.M) {
                    const uint8_t* p = sc + (int64_t)(R >> 4) * 16 * nblk + grp * 128 + (R & 15) * w;
                    if (w == 8) {
                        const uint2 v = __ldg(reinterpret_cast<const uint2*>(p));
                        rw[q][0] = v.x;
                        rw[q][1] = v.y;
                    } else {
                        for (int b = 0; b < w; ++b) rw[q][b >> 2] |= (uint32_t)__ldg(p + b) << (8 * (b & 3));
                    }
                }
            }
            uint32_t tw[2][4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const bool in = 32 * j + lane < item.n;
                const uint32_t* src = a.bsf + (int64_t)(item.g0 + 32 * j + lane) * nst + 2 * grp;
                tw[0][j] = in ? __ldg(src) : 0u;
                tw[1][j] = (in && w > 4) ? __ldg(src + 1) : 0u;
            }
            if (!warp_wait(&sh.abort, &sh.empty[slot], ((g / kS2) & 1) ^ 1, status, 8u)) return;
            char* Sa = smem + slot * kS2Slot + kS2A + kS2B;
            char* Sb = Sa + kS2Sa;
#pragma unroll
            for (int s = 0; s < 2; ++s) {
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    *reinterpret_cast<uint4*>(Sa + s * kM * 16 + (4 * lane + q) * 16) =
                        make_uint4(rw[q][s], rw[q][s], rw[q][s], rw[q][s]);
                *reinterpret_cast<uint4*>(Sb + s * 512 + lane * 16) = make_uint4(tw[s][0], tw[s][1], tw[s][2], tw[s][3]);
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) bar_arrive(&sh.full[slot]);
        }
    }
}

// MMA issuer (warp 14): per stage the scale copies, then w MMAs of K = 32;
// MMA k reads byte k & 3 of scale column (k >> 2) of the stage.
__device__ __forceinline__ void role_mma_mx2(Shared& sh, const GroupedArgs& a, char* smem) {
    const int nblk = a.K >> 5, ngrp = (nblk + 7) >> 3;
    const int lane = threadIdx.x & 31;
    unsigned* status = a.w.status;
    const uint32_t base = saddr(smem);
    int g = 0, il = 0;
    bool ok = true;
    for (int it = blockIdx.x; ok && it < sh.nitems; it += gridDim.x, ++il) {
        const Item item = decode(sh, it);
        const int n = max(16, (item.n + 15) & ~15);
        // a E2M1 (5), b E4M3 (0), E8M0 scales, N, M = 128, K = 32
        const uint32_t idesc0 = (5u << 7) | (0u << 10) | (1u << 23) | ((uint32_t)(n >> 3) << 17) |
                                ((uint32_t)(kM >> 4) << 24);
        const int b = il & 1;
        if (!warp_wait(&sh.abort, &sh.tempty[b], ((il >> 1) & 1) ^ 1, status, 16u)) break;
        tc_after_sync();
        const uint32_t dtm = sh.tmem + b * kNMax;
        bool first = true;
        for (int grp = 0; grp < ngrp; ++grp, ++g) {
            const int w = min(8, nblk - 8 * grp);
            const int slot = g % kS2;
            if (!warp_wait(&sh.abort, &sh.full[slot], (g / kS2) & 1, status, 32u)) { ok = false; break; }
            tc_after_sync();
            if (lane == 0) {
                const uint32_t A = base + slot * kS2Slot, B = A + kS2A, Sa = B + kS2B, Sb = Sa + kS2Sa;
                const uint32_t sfa = sh.tmem + kS2Sfa + slot * 8, sfb = sh.tmem + kS2Sfb + slot * 8;
                for (int s = 0; s * 4 < w; ++s) {
                    tc_cp_128x128b(sfa + 4 * s, smem_desc(Sa + s * kM * 16, 128, 128, 0));
                    tc_cp_32x128b_x4(sfb + 4 * s, smem_desc(Sb + s * 512, 128, 128, 0));
                }
                for (int k = 0; k < w; ++k) {
                    const uint32_t idesc = idesc0 | ((uint32_t)(k & 3) << 29) | ((uint32_t)(k & 3) << 4);
                    const uint32_t off = (k >> 2) * (kS2A / 2) + (k & 3) * 32;
                    tc_mma_mx(dtm, smem_desc(A + off, 16, 1024, 2), smem_desc(B + off, 16, 1024, 2), idesc,
                              first ? 0u : 1u, sfa + 4 * (k >> 2), sfb + 4 * (k >> 2));
                    first = false;
                }
                tc_commit(&sh.empty[slot]);
            }
            __syncwarp();
        }
        if (!ok) break;
        if (lane == 0) tc_commit(&sh.tfull[b]);
        __syncwarp();
    }
    if (lane == 0) {
        tc_commit(&sh.fin);
        const long long t0 = clock64();
        while (!bar_try(&sh.fin, 0)) {
            if (clock64() - t0 > kWaitCycles) {
                if (status) atomicOr(status, 64u);
                break;
            }
        }
    }
    __syncwarp();
}

template <int kMode>
__global__ void __launch_bounds__(kThreads, 1) k_grouped(const __grid_constant__ CUtensorMap bmap,
                                                         GroupedArgs a) {
    extern __shared__ unsigned char dyn_raw[];
    __shared__ Shared sh;
    char* smem = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(dyn_raw) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x, warp = tid >> 5;

    if (tid == 0) {
        for (int i = 0; i < kStages; ++i) { bar_init(&sh.full[i], kConvWarps + 1); bar_init(&sh.empty[i], 1); }
        for (int i = 0; i < kGroups; ++i) { bar_init(&sh.gfull[i], 1); bar_init(&sh.gempty[i], kConvWarps); }
        for (int i = 0; i < 2; ++i) { bar_init(&sh.tfull[i], 1); bar_init(&sh.tempty[i], 128); }
        bar_init(&sh.fin, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    plan_items(sh, a);
    if (sh.nitems <= (int)blockIdx.x) return;  // no work for this CTA (uniform)
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(&sh.tmem)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_before_sync();
    __syncthreads();
    tc_after_sync();
    if (warp < kConvWarps) role_convert(sh, a, smem);
    else if (warp < kWeightWarp) role_epilogue<kMode, false>(sh, a);
    else if (warp == kWeightWarp) role_weights(sh, a, smem);
    else if (warp == kTokenWarp) role_tokens(sh, a, smem, &bmap);
    else role_mma(sh, a, smem);

    tc_before_sync();
    __syncthreads();
    tc_after_sync();
    // A CTA that gave up may still have bulk copies landing in its shared
    // memory: give them time (they complete in microseconds) before exiting.
    if (*(volatile int*)&sh.abort) {
        const long long t0 = clock64();
        while (clock64() - t0 < 2000000) {}
    }
    if (warp == kMmaWarp)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(sh.tmem), "r"(kTmemCols)
                     : "memory");
}

// The block-scaled grouped GEMM (roles above role_copies_mx2).  Warps 0-7
// have no role in this mode.
template <int kMode>
__global__ void __launch_bounds__(kThreads, 1) k_grouped_mx(const __grid_constant__ MxMaps maps, GroupedArgs a) {
    extern __shared__ unsigned char dyn_raw[];
    __shared__ Shared sh;
    char* smem = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(dyn_raw) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x, warp = tid >> 5;
    if (tid == 0) {
        // full: the copies' transaction count plus the scale warp's arrival
        for (int i = 0; i < kS2; ++i) { bar_init(&sh.full[i], 2); bar_init(&sh.empty[i], 1); }
        for (int i = 0; i < 2; ++i) { bar_init(&sh.tfull[i], 1); bar_init(&sh.tempty[i], 128); }
        bar_init(&sh.fin, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    plan_items(sh, a);
    if (sh.nitems <= (int)blockIdx.x) return;  // no work for this CTA (uniform)
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(&sh.tmem)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_before_sync();
    __syncthreads();
    tc_after_sync();
    if (warp >= kEpiWarp0 && warp < kWeightWarp) role_epilogue<kMode, true>(sh, a);
    else if (warp == kWeightWarp) {
        if ((tid & 31) == 0) role_copies_mx2(sh, a, smem, &maps);
        __syncwarp();
    } else if (warp == kTokenWarp) role_scales_mx2(sh, a, smem);
    else if (warp == kMmaWarp) role_mma_mx2(sh, a, smem);

    tc_before_sync();
    __syncthreads();
    tc_after_sync();
    // A CTA that gave up may still have copies landing in its shared memory:
    // give them time (they complete in microseconds) before exiting.
    if (*(volatile int*)&sh.abort) {
        const long long t0 = clock64();
        while (clock64() - t0 < 2000000) {}
    }
    if (warp == kMmaWarp)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(sh.tmem), "r"(kTmemCols)
                     : "memory");
}

// x16 rows in expert order: row epre[e] + i = x16[list[e][i] / k] (epre the
// exclusive prefix of the experts' token counts).  grid (E, 32), 256 threads.
__global__ void __launch_bounds__(256) k_gather(MoeDims d, MoeWork w, int H) {
    __shared__ int off;
    const int e = blockIdx.x;
    if (threadIdx.x < 32) {
        int s = 0;
        for (int j = threadIdx.x; j < e; j += 32) s += min(w.counts[j], w.tcap);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (threadIdx.x == 0) off = s;
    }
    __syncthreads();
    const int cnt = min(w.counts[e], w.tcap);
    const int chunks = H >> 3;  // 16-byte pieces per row
    for (int i = blockIdx.y; i < cnt; i += gridDim.y) {
        const int tok = w.lists[(int64_t)e * w.tcap + i] / d.k;
        const uint4* src = reinterpret_cast<const uint4*>(w.x16 + (int64_t)tok * H);
        uint4* dst = reinterpret_cast<uint4*>(w.xg + (int64_t)(off + i) * H);
        for (int c = threadIdx.x; c < chunks; c += blockDim.x) dst[c] = src[c];
    }
}

// One row of K values -> MXFP8: E4M3 codes q[K] and scale words sf[ceil(K/128)]
// (byte b of word s = the E8M0 scale of block 4s + b).  One warp; lane l
// takes values 4l..4l+3 of each 128-value stage, 8 lanes per 32-value block.
// Scale = 2^(floor(log2 max|x|) - 8) (byte = the max's biased exponent - 8,
// clamped to [0, 254]; 0 for an all-zero block); codes = x / scale rounded to
// nearest-even E4M3, saturating.  oracle.quantize_mxfp8 restates this.
template <typename In>
__device__ __forceinline__ void quantize_row_mx(const In* __restrict__ src, int K, uint8_t* __restrict__ q,
                                                uint32_t* __restrict__ sf) {
    const int lane = threadIdx.x & 31;
    const int nst = (K + 127) >> 7;
    for (int s = 0; s < nst; ++s) {
        const int c = s * 128 + lane * 4;
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        if (c < K) {
            const uint2 raw = *reinterpret_cast<const uint2*>(src + c);
            const uint32_t u[2] = {raw.x, raw.y};
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                if constexpr (sizeof(In) == 2 && std::is_same<In, __half>::value) {
                    const __half2 h = *reinterpret_cast<const __half2*>(&u[j]);
                    v[2 * j] = __low2float(h);
                    v[2 * j + 1] = __high2float(h);
                } else {  // bf16 bits
                    v[2 * j] = __uint_as_float(u[j] << 16);
                    v[2 * j + 1] = __uint_as_float(u[j] & 0xffff0000u);
                }
            }
        }
        float m = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
        const int eb = (int)((__float_as_uint(m) >> 23) & 0xffu);
        const int byte = m > 0.f ? min(254, max(0, eb - 8)) : 0;
        const int p = 127 - byte, p1 = p / 2;
        const float f1 = pow2f(p1), f2 = pow2f(p - p1);
        uint32_t lo, hi;
        asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(*reinterpret_cast<unsigned short*>(&lo)) : "f"(v[1] * f1 * f2), "f"(v[0] * f1 * f2));
        asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(*reinterpret_cast<unsigned short*>(&hi)) : "f"(v[3] * f1 * f2), "f"(v[2] * f1 * f2));
        if (c < K) *reinterpret_cast<uint32_t*>(q + c) = (lo & 0xffffu) | ((hi & 0xffffu) << 16);
        const uint32_t b0 = __shfl_sync(0xffffffffu, byte, 0), b1 = __shfl_sync(0xffffffffu, byte, 8);
        const uint32_t b2 = __shfl_sync(0xffffffffu, byte, 16), b3 = __shfl_sync(0xffffffffu, byte, 24);
        if (lane == 0) sf[s] = b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
    }
}

// Block-scaled mode's token rows: every (expert, token) slot's x row quantised
// to MXFP8 in expert order (row epre[e] + i).  grid (E, 32), 8 warps.
template <typename In>
__global__ void __launch_bounds__(256) k_gather_mx(MoeDims d, MoeWork w, const In* __restrict__ x, int H) {
    __shared__ int off;
    const int e = blockIdx.x, warp = threadIdx.x >> 5;
    if (threadIdx.x < 32) {
        int s = 0;
        for (int j = threadIdx.x; j < e; j += 32) s += min(w.counts[j], w.tcap);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (threadIdx.x == 0) off = s;
    }
    __syncthreads();
    const int cnt = min(w.counts[e], w.tcap), nst = (H + 127) >> 7;
    for (int i = blockIdx.y * 8 + warp; i < cnt; i += gridDim.y * 8) {
        const int tok = w.lists[(int64_t)e * w.tcap + i] / d.k;
        quantize_row_mx(x + (int64_t)tok * H, H, w.xq + (int64_t)(off + i) * H, w.xsf + (int64_t)(off + i) * nst);
    }
}

// Block-scaled mode's activations: the f16 rows gate_up wrote (expert order)
// quantised to MXFP8 for the down projection.  One warp per row.
__global__ void __launch_bounds__(256) k_quant_act(MoeWork w, int rows, int F) {
    const int r = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (r >= rows) return;
    const int nst = (F + 127) >> 7;
    quantize_row_mx(w.act + (int64_t)r * F, F, w.aq + (int64_t)r * F, w.asf + (int64_t)r * nst);
}

// Largest E8M0 exponent of each row (bytes 1..254; 127 when the row has
// none) of a row-major scale matrix.
__global__ void k_rowexp(const uint8_t* __restrict__ scales, int rows, int nblk, uint8_t* __restrict__ out) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    int m = 0;
    for (int b = 0; b < nblk; ++b) {
        const int v = scales[(int64_t)r * nblk + b];
        if (v != 0 && v != 255 && v > m) m = v;
    }
    out[r] = (uint8_t)(m == 0 ? 127 : m);
}

}  // namespace

// cuTensorMapEncodeTiled from the driver, resolved once (nullptr if absent).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}


int configure_grouped() {
    const void* fns[3] = {(const void*)k_grouped<0>, (const void*)k_grouped<1>, (const void*)k_grouped<2>};
    for (const void* f : fns)
        if (cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, kDynSmem) != cudaSuccess) return -1;
    const void* mx[3] = {(const void*)k_grouped_mx<0>, (const void*)k_grouped_mx<1>, (const void*)k_grouped_mx<2>};
    for (const void* f : mx)
        if (cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, kS2Smem) != cudaSuccess) return -1;
    return 0;
}

namespace {
// The block-scaled kernel's two 4-bit views of one matrix of the layer's bank
// (tiled layout: 16-row tiles, 8-block groups of 16 rows x 128 bytes, the
// last group 16 rows x 16 w bytes; experts one stride apart).
bool encode_weight_maps(MxMaps& m, const LayerView& L, int sec_packed, int M, int K, int e_local) {
    auto enc = tensor_map_encoder();
    if (!enc) return false;
    const int nblk = K / 32, nfull = nblk / 8, ntiles = M / 16;
    const int w = nblk - 8 * nfull;  // blocks of the last, narrow group (0: none)
    const uint8_t* pk = L.base + L.off[sec_packed];
    const cuuint64_t tile_pk = (cuuint64_t)nblk * 256, es = (cuuint64_t)L.stride;
    const cuuint32_t ones[5] = {1, 1, 1, 1, 1};
    {
        const cuuint64_t gd[5] = {256, 16, (cuuint64_t)(nfull > 0 ? nfull : 1), (cuuint64_t)ntiles, (cuuint64_t)e_local};
        const cuuint64_t gs[4] = {128, 2048, tile_pk, es};
        const cuuint32_t box[5] = {128, 16, 1, 8, 1};
        if (enc(&m.wfull, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 5, const_cast<uint8_t*>(pk), gd, gs, box, ones,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    }
    {
        // the last group's rows are 16 w bytes apart; its 128-value box reads
        // zeros past the row (or, where the driver wants the box inside the
        // view, the next row's codes), which the stage's w MMAs never use
        const int wn = w > 0 ? w : 8;
        const cuuint64_t gs[3] = {(cuuint64_t)(16 * wn), tile_pk, es};
        const cuuint32_t box[4] = {128, 16, 8, 1};
        uint8_t* nb = const_cast<uint8_t*>(pk + (w > 0 ? (int64_t)nfull * 2048 : 0));
        bool ok = false;
        for (cuuint64_t d0 : {(cuuint64_t)(32 * wn), (cuuint64_t)128}) {
            const cuuint64_t gd[4] = {d0, 16, (cuuint64_t)ntiles, (cuuint64_t)e_local};
            if (enc(&m.wnarrow, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 4, nb, gd, gs, box, ones,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS) {
                ok = true;
                break;
            }
        }
        if (!ok) return false;
    }
    return true;
}
}  // namespace

bool grouped_supported(const MoeDims& d, const MoeWork& w) {
    // an even number of 32-column blocks per row (stages of 4 or 2 blocks);
    // rows of both matrices are multiples of 16 (bank creation requires
    // multiples of 32 for H and F)
    return w.status != nullptr && d.H % 64 == 0 && d.F % 64 == 0 && tensor_map_encoder() != nullptr;
}

int launch_grouped(const LayerView& L, const MoeDims& d, const MoeWork& w, int which, int sms,
                   cudaStream_t s, const void* x, int x_dtype) {
    const bool mx = w.block_scaled != 0;
    if (mx && which == 0 && !x) return -1;  // the block-scaled gather quantises the layer input
    GroupedArgs a;
    a.L = L;
    a.d = d;
    a.w = w;
    const void* bsrc;
    uint64_t brows = (uint64_t)w.tcap * d.k;
    if (which == 0) {
        a.M = 2 * d.F; a.K = d.H;
        a.sec_packed = 0; a.sec_scales = 1; a.sec_bias = 4;
        a.rexp_off = 0;
        bsrc = mx ? (const void*)w.xq : (const void*)w.xg;
        a.bsf = w.xsf;
        a.bdiv = d.k;
        a.mode = d.act == 0 ? 0 : 1;
    } else {
        a.M = d.H; a.K = d.F;
        a.sec_packed = 2; a.sec_scales = 3; a.sec_bias = 5;
        a.rexp_off = 2 * d.F;
        bsrc = mx ? (const void*)w.aq : (const void*)w.act;
        a.bsf = w.asf;
        a.bdiv = 1;
        a.mode = 2;
    }
    // expert-ordered token rows [brows][K] (f16, or E4M3 codes in the
    // block-scaled mode), one 128-byte row slice x 128 rows per box, 128-byte
    // swizzle
    CUtensorMap map;
    const int esz = mx ? 1 : 2;
    const cuuint64_t gdim[2] = {(cuuint64_t)a.K, brows};
    const cuuint64_t gstride[1] = {(cuuint64_t)a.K * esz};
    const cuuint32_t box[2] = {(cuuint32_t)(128 / esz), kNMax}, estride[2] = {1, 1};
    auto enc = tensor_map_encoder();
    if (!enc || enc(&map, mx ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                    const_cast<void*>(bsrc), gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return -1;
    int launched = 0;
    if (which == 0) {
        if (!mx) k_gather<<<dim3(d.E, 32), 256, 0, s>>>(d, w, d.H);
        else if (x_dtype == kF16) k_gather_mx<__half><<<dim3(d.E, 32), 256, 0, s>>>(d, w, static_cast<const __half*>(x), d.H);
        else k_gather_mx<uint16_t><<<dim3(d.E, 32), 256, 0, s>>>(d, w, static_cast<const uint16_t*>(x), d.H);
        ++launched;
    } else if (mx) {
        const int rows = w.tcap * d.k;
        k_quant_act<<<(rows + 7) / 8, 256, 0, s>>>(w, rows, d.F);
        ++launched;
    }
    const dim3 grid(sms), block(kThreads);
    if (mx) {
        MxMaps maps;
        const cuuint32_t box32[2] = {128, 32};
        if (enc(&maps.b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(bsrc), gdim, gstride, box32, estride,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return -1;
        const int e_local = (d.E - d.shard_rank + d.shard_count - 1) / d.shard_count;
        if (!encode_weight_maps(maps, L, a.sec_packed, a.M, a.K, e_local)) return -1;
        if (a.mode == 0) k_grouped_mx<0><<<grid, block, kS2Smem, s>>>(maps, a);
        else if (a.mode == 1) k_grouped_mx<1><<<grid, block, kS2Smem, s>>>(maps, a);
        else k_grouped_mx<2><<<grid, block, kS2Smem, s>>>(maps, a);
    } else {
        if (a.mode == 0) k_grouped<0><<<grid, block, kDynSmem, s>>>(map, a);
        else if (a.mode == 1) k_grouped<1><<<grid, block, kDynSmem, s>>>(map, a);
        else k_grouped<2><<<grid, block, kDynSmem, s>>>(map, a);
    }
    return cudaGetLastError() == cudaSuccess ? launched + 1 : -1;
}

int launch_rowexp(const uint8_t* scales, int rows, int cols, uint8_t* out, cudaStream_t s) {
    k_rowexp<<<(rows + 127) / 128, 128, 0, s>>>(scales, rows, cols >> 5, out);
    return cudaGetLastError() == cudaSuccess ? 1 : -1;
}


}  // namespace gw
