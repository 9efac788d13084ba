// gw_device.cuh — device helpers shared by the sm_100a kernels.
//
// MXFP4 weights stay packed in HBM exactly as the reference installs them
// (Install/InstallLayout.swift:56-91: row-major [rows][cols/2] nibbles, low
// nibble = even column; one E8M0 scale byte per 32-column block).  The GEMV
// core converts nibble pairs straight into f16x2 tensor-core fragments with
// the sm_100a `cvt.rn.f16x2.e2m1x2` instruction and multiplies them against
// f16 activations with `mma.sync.m16n8k16` (fp32 accumulate), one 32-column
// block at a time, then scales the block's fp32 partial by its E8M0 scale —
// the same "partial per block, then acc += partial * scale" structure as the
// reference's GEMVs (Metal/Quant/dequant_gemv.metal:50-63).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace gw {

constexpr int kWarp = 32;

// E8M0 scale as the reference GPU kernels decode it: exp2(byte - 127)
// (Metal/Quant/dequant_gemv.metal:30-32).  For bytes 1..254 the fp32 bit
// pattern byte<<23 is exactly 2^(byte-127); byte 255 gives +inf (exp2(128)),
// byte 0 gives 0 (the Metal build runs with fast math, which flushes the
// 2^-127 denormal).  The bit-exact dequant kernel uses the CPU decoder's rule
// instead (see decode_scale_exact).
__device__ __forceinline__ float gemv_scale(uint32_t byte) {
    return __uint_as_float(byte << 23);
}

// MXFP4.decodeScale (Quant/MXFP4.swift:37-40): NaN for 0xFF, 2^(byte-127)
// otherwise, including the 2^-127 denormal for byte 0.
__device__ __forceinline__ float decode_scale_exact(uint32_t byte) {
    if (byte == 0xFFu) return __uint_as_float(0x7FC00000u);
    if (byte == 0u) return __uint_as_float(0x00400000u);
    return __uint_as_float(byte << 23);
}

// Four packed bytes (eight E2M1 codes) -> four f16x2 registers, register i
// holding byte i's low nibble in its low half.
__device__ __forceinline__ void e2m1x8_to_f16x8(uint32_t w, uint32_t& r0, uint32_t& r1,
                                                uint32_t& r2, uint32_t& r3) {
    asm("{\n\t"
        ".reg .b8 q0, q1, q2, q3;\n\t"
        "mov.b32 {q0, q1, q2, q3}, %4;\n\t"
        "cvt.rn.f16x2.e2m1x2 %0, q0;\n\t"
        "cvt.rn.f16x2.e2m1x2 %1, q1;\n\t"
        "cvt.rn.f16x2.e2m1x2 %2, q2;\n\t"
        "cvt.rn.f16x2.e2m1x2 %3, q3;\n\t"
        "}"
        : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
        : "r"(w));
}

// D = A(16x16 f16, row) * B(16x8 f16, col) + C, fp32 accumulate.
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1,
                                         const float (&c)[4]) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%10, %11, %12, %13};\n"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]),
          "f"(c[2]), "f"(c[3]));
}

__device__ __forceinline__ uint32_t ldg_u32(const uint32_t* p) { return __ldg(p); }

// Starts an L2 fill of [p, p + bytes) (both 16-byte aligned, bytes a multiple
// of 16) without holding registers or shared memory: the later loads of the
// range then wait on L2, not on DRAM.
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ uint32_t ldg_u8(const uint8_t* p) {
    return static_cast<uint32_t>(__ldg(p));
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t v) {
    return __uint_as_float(static_cast<uint32_t>(v) << 16);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// ---------------------------------------------------------------------------
// Block-diagonal MXFP4 tile: one warp, 16 weight rows (rowA / rowB halves),
// blocks [blk0, blk1), 1..8 tokens.
//
// Each thread streams WHOLE 16-byte blocks with 128-bit loads: in round r of
// an 8-block group, thread t of a quad owns block base + 4r + t of rows rowA
// and rowB, so a warp load covers 64 contiguous bytes of 8 rows (full
// sectors).  The four threads of an MMA quad therefore feed four different
// blocks (four different scales) into one m16n8k16 MMA, so each block's
// partial is kept apart by the B operand: the B fragment of thread (g, t)
// holds x[token][that thread's block] only when column g belongs to
// (block t, token) and zeros otherwise (a shared zero block).  D[row][col]
// then accumulates exactly one (block, token) partial per column, which is
// scaled by its E8M0 scale (and the x block scale) into fp32 accumulators —
// the reference's "acc += partial * scale" — before the MMA accumulator
// restarts from zero.
//
//   kTok = 1: columns = the 8 blocks of the group (one token).
//   kTok = 2: columns = 4 blocks x 2 tokens; kSets token pairs share each
//             converted weight fragment (their MMAs use separate
//             accumulators), so 2*kSets tokens cost one weight conversion.
//
// Shared x layout: xs[token][block][40 halves] (32 values + 8 pad, which
// keeps the four active threads' 16-byte loads on distinct banks); the block
// at index `zero_blk` of token row 0 is all zeros.  The results are in the
// units of the staged x (the caller applies the token's x scale).
constexpr int kXBlockHalves = 40;

// Weight layouts the tile can stream:
//   kTiled = false: the reference's row-major layout; rowA / rowB are matrix
//     rows and packed / scales the matrix base.
//   kTiled = true: the bank's tiled layout (see tile_layout_offset); rowA /
//     rowB are rows 0..15 of the tile and packed / scales point at the tile.
//   kPrefetch (tiled layout only): 1 = start an L2 fill of the warp's whole
//     K-range up front (measured on B200: ~10% faster gate_up GEMVs at decode
//     batch 64, slightly slower down GEMVs and batch 1); D >= 2 = keep the L2
//     fill D 8-block groups ahead of the loads; 0 = none.
template <int kTok, int kSets, bool kTiled = false, int kPrefetch = 0>
__device__ __forceinline__ void mxfp4_tile_diag(const uint8_t* __restrict__ packed,
                                                const uint8_t* __restrict__ scales, int cols,
                                                int rowA, int rowB, const __half* xs,
                                                int xs_stride, int ntok,
                                                int blk0, int blk1,
                                                float (&accA)[kTok * kSets],
                                                float (&accB)[kTok * kSets]) {
    static_assert((kTok == 1 && kSets == 1) || kTok == 2, "1 token, or token pairs");
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int nblk = blk1;
    const int row_blocks = cols >> 5;
    const int zero_blk = row_blocks;  // the zero block
    const size_t rb = (size_t)(cols >> 1);
    const uint4* pA = reinterpret_cast<const uint4*>(packed + (kTiled ? 0 : (size_t)rowA * rb));
    const uint4* pB = reinterpret_cast<const uint4*>(packed + (kTiled ? 0 : (size_t)rowB * rb));
    const uint8_t* sA = scales + (kTiled ? 0 : (size_t)rowA * row_blocks);
    const uint8_t* sB = scales + (kTiled ? 0 : (size_t)rowB * row_blocks);
#pragma unroll
    for (int j = 0; j < kTok * kSets; ++j) { accA[j] = 0.f; accB[j] = 0.f; }
    // Put the warp's whole K-range in flight at once (the register loads below
    // keep only one 8-block group ahead): in the tiled layout blocks
    // [blk0, blk1) of the tile's 16 rows are one contiguous run of groups.
    const uint32_t tile_pk = 16u * (uint32_t)(cols >> 1), tile_sc = 16u * (uint32_t)(cols >> 5);
    if (kPrefetch && kTiled && blk1 > blk0) {
        {
            const int blk_end = kPrefetch == 1 ? blk1 : min(blk1, blk0 + 8 * (kPrefetch + 1));
            if (lane == 0) {
                const uint32_t lo = (uint32_t)(blk0 >> 3) * 2048u;
                const uint32_t hi = min((uint32_t)((blk_end + 7) >> 3) * 2048u, tile_pk);
                prefetch_l2_bulk(packed + lo, hi - lo);
            } else if (lane == 1) {  // the groups' scale bytes (16 rows x w per group)
                const uint32_t lo = (uint32_t)(blk0 >> 3) * 128u;
                const uint32_t hi = min((uint32_t)((blk_end + 7) >> 3) * 128u, tile_sc);
                prefetch_l2_bulk(scales + lo, hi - lo);
            }
        }
    }

    // Per 8-block group: the group's first block of row A / row B, and its
    // width in the layout (the tiled layout stores a group's rows w blocks
    // apart; the row-major layout keeps the row's own stride).
    auto group_ptrs = [&](int base, const uint4*& gA, const uint4*& gB, const uint8_t*& hA,
                          const uint8_t*& hB) {
        if (kTiled) {
            const int w = min(8, row_blocks - base);
            const size_t g0 = (size_t)(base >> 3) * 128;
            gA = pA + g0 + rowA * w; gB = pB + g0 + rowB * w;
            hA = sA + g0 + rowA * w; hB = sB + g0 + rowB * w;
        } else {
            gA = pA + base; gB = pB + base; hA = sA + base; hB = sB + base;
        }
    };
    uint4 wa[2], wb[2];
    auto load = [&](int base) {
        const uint4 *gA, *gB;
        const uint8_t *hA, *hB;
        group_ptrs(base, gA, gB, hA, hB);
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int j = 4 * r + t;
            if (base + j < nblk) { wa[r] = __ldg(gA + j); wb[r] = __ldg(gB + j); }
            else { wa[r] = make_uint4(0, 0, 0, 0); wb[r] = make_uint4(0, 0, 0, 0); }
        }
    };
    // x source of this thread's B fragment for (round r, set s): the token
    // row and block when column g is (this thread's block, token), else the
    // zero block.
    auto xsrc = [&](int r, int s, int base) -> const uint4* {
        const int blk = base + 4 * r + t;
        int tok = -1;
        if (kTok == 1) tok = (g == 4 * r + t) ? 0 : -1;
        else tok = (g >> 1) == t ? 2 * s + (g & 1) : -1;
        const bool live = tok >= 0 && tok < ntok && blk < nblk;
        return reinterpret_cast<const uint4*>(live ? xs + tok * xs_stride + blk * kXBlockHalves
                                                   : xs + zero_blk * kXBlockHalves);
    };
    load(blk0);
    for (int base = blk0; base < nblk; base += 8) {
        const uint4 *gA_, *gB_;
        const uint8_t *hA, *hB;
        group_ptrs(base, gA_, gB_, hA, hB);
        uint4 ca[2], cb[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) { ca[r] = wa[r]; cb[r] = wb[r]; }
        if (base + 8 < nblk) load(base + 8);  // next group's loads in flight
        if (kPrefetch >= 2 && kTiled && lane < 2) {  // the group kPrefetch + 1 ahead, into L2
            const int nb = base + 8 * (kPrefetch + 1);
            if (nb < nblk) {
                const uint32_t unit = lane == 0 ? 2048u : 128u, total = lane == 0 ? tile_pk : tile_sc;
                const uint32_t lo = (uint32_t)(nb >> 3) * unit;
                prefetch_l2_bulk((lane == 0 ? packed : scales) + lo, min(unit, total - lo));
            }
        }
        float d[kSets][4];
#pragma unroll
        for (int s = 0; s < kSets; ++s) d[s][0] = d[s][1] = d[s][2] = d[s][3] = 0.f;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const uint4* xp[kSets];
#pragma unroll
            for (int s = 0; s < kSets; ++s) xp[s] = xsrc(r, s, base);
            const uint32_t wA[4] = {ca[r].x, ca[r].y, ca[r].z, ca[r].w};
            const uint32_t wB[4] = {cb[r].x, cb[r].y, cb[r].z, cb[r].w};
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                uint32_t a0, a1, a2, a3, q0, q1, q2, q3;
                e2m1x8_to_f16x8(wA[w], a0, a1, a2, a3);
                e2m1x8_to_f16x8(wB[w], q0, q1, q2, q3);
#pragma unroll
                for (int s = 0; s < kSets; ++s) {
                    const uint4 xv = xp[s][w];
                    // step 2w: bytes 0,1 of word w; step 2w+1: bytes 2,3
                    mma16816(d[s], a0, q0, a1, q1, xv.x, xv.y, d[s]);
                    mma16816(d[s], a2, q2, a3, q3, xv.z, xv.w, d[s]);
                }
            }
            if constexpr (kTok == 2) {
                // flush this round: column 2t+q = (block base+4r+t, token 2s+q)
                const int blk = base + 4 * r + t;
                const bool ok = blk < nblk;
                const float fa = ok ? gemv_scale(ldg_u8(hA + 4 * r + t)) : 0.f;
                const float fb = ok ? gemv_scale(ldg_u8(hB + 4 * r + t)) : 0.f;
#pragma unroll
                for (int s = 0; s < kSets; ++s) {
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        const int tok = 2 * s + q;
                        accA[tok] = fmaf(d[s][q], fa, accA[tok]);
                        accB[tok] = fmaf(d[s][2 + q], fb, accB[tok]);
                    }
                    d[s][0] = d[s][1] = d[s][2] = d[s][3] = 0.f;
                }
            }
        }
        if constexpr (kTok == 1) {
            // flush the group: column 2t+q = block base+2t+q
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const int blk = base + 2 * t + q;
                const bool ok = blk < nblk;
                const float fa = ok ? gemv_scale(ldg_u8(hA + 2 * t + q)) : 0.f;
                const float fb = ok ? gemv_scale(ldg_u8(hB + 2 * t + q)) : 0.f;
                accA[0] = fmaf(d[0][q], fa, accA[0]);
                accB[0] = fmaf(d[0][2 + q], fb, accB[0]);
            }
        }
    }
    // sum the quad's columns
#pragma unroll
    for (int j = 0; j < kTok * kSets; ++j) {
        accA[j] += __shfl_xor_sync(0xffffffffu, accA[j], 1);
        accA[j] += __shfl_xor_sync(0xffffffffu, accA[j], 2);
        accB[j] += __shfl_xor_sync(0xffffffffu, accB[j], 1);
        accB[j] += __shfl_xor_sync(0xffffffffu, accB[j], 2);
    }
}

// One 8-block group of mxfp4_tile_diag, for weights already in shared
// memory (or any generic address): gA / gB point at the group's first block
// of rows A and B (w blocks per row, the group's width), hA / hB at their
// scale bytes; base = the group's first block in the row, nblk = the row's
// blocks (the zero block of xs sits at index nblk).  Accumulates into
// accA / accB the same per-block partials times scales as one iteration of
// mxfp4_tile_diag's group loop, with the partials summed over four
// independent MMA chains; the caller sums the quad at the end (quad_sum_acc).
template <int kTok, int kSets>
__device__ __forceinline__ void mxfp4_group_diag(const uint4* gA, const uint4* gB, const uint8_t* hA,
                                                 const uint8_t* hB, int base, int nblk, const __half* xs,
                                                 int xs_stride, int ntok, float (&accA)[kTok * kSets],
                                                 float (&accB)[kTok * kSets]) {
    static_assert((kTok == 1 && kSets == 1) || kTok == 2, "1 token, or token pairs");
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int zero_blk = nblk;
    uint4 ca[2], cb[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int j = 4 * r + t;
        if (base + j < nblk) { ca[r] = gA[j]; cb[r] = gB[j]; }
        else { ca[r] = make_uint4(0, 0, 0, 0); cb[r] = make_uint4(0, 0, 0, 0); }
    }
    auto xsrc = [&](int r, int s) -> const uint4* {
        const int blk = base + 4 * r + t;
        int tok = -1;
        if (kTok == 1) tok = (g == 4 * r + t) ? 0 : -1;
        else tok = (g >> 1) == t ? 2 * s + (g & 1) : -1;
        const bool live = tok >= 0 && tok < ntok && blk < nblk;
        return reinterpret_cast<const uint4*>(live ? xs + tok * xs_stride + blk * kXBlockHalves
                                                   : xs + zero_blk * kXBlockHalves);
    };
    // four independent MMA chains per token set (round r, even / odd word)
    // so a warp keeps several MMAs in flight; summed before each flush
    float d[2][kSets][2][4];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int s = 0; s < kSets; ++s)
#pragma unroll
            for (int h = 0; h < 2; ++h) d[r][s][h][0] = d[r][s][h][1] = d[r][s][h][2] = d[r][s][h][3] = 0.f;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const uint4* xp[kSets];
#pragma unroll
        for (int s = 0; s < kSets; ++s) xp[s] = xsrc(r, s);
        const uint32_t wA[4] = {ca[r].x, ca[r].y, ca[r].z, ca[r].w};
        const uint32_t wB[4] = {cb[r].x, cb[r].y, cb[r].z, cb[r].w};
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            uint32_t a0, a1, a2, a3, q0, q1, q2, q3;
            e2m1x8_to_f16x8(wA[w], a0, a1, a2, a3);
            e2m1x8_to_f16x8(wB[w], q0, q1, q2, q3);
#pragma unroll
            for (int s = 0; s < kSets; ++s) {
                const uint4 xv = xp[s][w];
                float(&dd)[4] = d[r][s][w & 1];
                mma16816(dd, a0, q0, a1, q1, xv.x, xv.y, dd);
                mma16816(dd, a2, q2, a3, q3, xv.z, xv.w, dd);
            }
        }
    }
    if constexpr (kTok == 2) {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int blk = base + 4 * r + t;
            const bool ok = blk < nblk;
            const float fa = ok ? gemv_scale(hA[4 * r + t]) : 0.f;
            const float fb = ok ? gemv_scale(hB[4 * r + t]) : 0.f;
#pragma unroll
            for (int s = 0; s < kSets; ++s) {
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    const int tok = 2 * s + q;
                    accA[tok] = fmaf(d[r][s][0][q] + d[r][s][1][q], fa, accA[tok]);
                    accB[tok] = fmaf(d[r][s][0][2 + q] + d[r][s][1][2 + q], fb, accB[tok]);
                }
            }
        }
    } else {
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const int blk = base + 2 * t + q;
            const bool ok = blk < nblk;
            const float fa = ok ? gemv_scale(hA[2 * t + q]) : 0.f;
            const float fb = ok ? gemv_scale(hB[2 * t + q]) : 0.f;
            const float sa = (d[0][0][0][q] + d[0][0][1][q]) + (d[1][0][0][q] + d[1][0][1][q]);
            const float sb = (d[0][0][0][2 + q] + d[0][0][1][2 + q]) + (d[1][0][0][2 + q] + d[1][0][1][2 + q]);
            accA[0] = fmaf(sa, fa, accA[0]);
            accB[0] = fmaf(sb, fb, accB[0]);
        }
    }
}

template <int kN>
__device__ __forceinline__ void quad_sum_acc(float (&accA)[kN], float (&accB)[kN]) {
#pragma unroll
    for (int j = 0; j < kN; ++j) {
        accA[j] += __shfl_xor_sync(0xffffffffu, accA[j], 1);
        accA[j] += __shfl_xor_sync(0xffffffffu, accA[j], 2);
        accB[j] += __shfl_xor_sync(0xffffffffu, accB[j], 1);
        accB[j] += __shfl_xor_sync(0xffffffffu, accB[j], 2);
    }
}

// Tiled bank layout of an MXFP4 matrix [rows][cols] (rows % 16 == 0): the
// 16-row tiles follow one another; inside a tile the 32-column blocks go in
// groups of 8 (the last group narrower), and each group stores its 16 rows
// x w blocks row-major.  A warp's pass over one group of its tile is thus one
// contiguous 2 KB read, and a tile streams from HBM front to back (the
// reference's row-major layout makes it 16 interleaved 128-byte-wide streams,
// which DRAM serves measurably worse).  Scale bytes follow the same scheme
// with 1-byte elements.  Returns the element offset of (row, blk).
__host__ __device__ __forceinline__ int64_t tile_layout_offset(int row, int blk, int nblk) {
    const int tile = row >> 4, lr = row & 15, grp = blk >> 3;
    const int w = (nblk - (grp << 3)) < 8 ? (nblk - (grp << 3)) : 8;
    return (int64_t)tile * 16 * nblk + (int64_t)grp * 128 + lr * w + (blk & 7);
}

// Expert activation on one (gate, up) pair, kAct 0 = clamped GLU, 1 = SiLU.
template <int kAct>
__device__ __forceinline__ float activate(float gate, float up, float limit, float alpha) {
    if (kAct == 0) {  // gptoss_expert_activation, expert.metal:92-101
        gate = fminf(gate, limit);
        up = fminf(fmaxf(up, -limit), limit);
        const float glu = gate * (1.0f / (1.0f + expf(-alpha * gate)));
        return (up + 1.0f) * glu;
    } else {  // expert_activation_swiglu, expert.metal:388-392
        const float silu = gate * (1.0f / (1.0f + expf(-gate)));
        return silu * up;
    }
}

// 2^p as an fp32 bit pattern, |p| <= 126.
__device__ __forceinline__ float pow2f(int p) { return __uint_as_float((uint32_t)(127 + p) << 23); }

// Shift p that brings a row maximum m into [2^15, 2^16): every bf16 value
// within 2^-24 of the row maximum then converts to f16 exactly after
// multiplying by 2^p, and the GEMV result is multiplied by 2^-p.  0 for zero
// or non-finite m.
__device__ __forceinline__ int row_exponent_shift(float m) {
    const uint32_t e = (__float_as_uint(m) >> 23) & 0xffu;  // biased exponent of m
    if (m == 0.f || e == 0xffu) return 0;
    const int ex = (e == 0 ? -126 : (int)e - 126);          // m < 2^ex
    const int p = 16 - ex;
    return p < -120 ? -120 : (p > 120 ? 120 : p);
}

// Stages n f16 rows (row_ids into src [*][cols]) into the padded block
// layout of mxfp4_tile_diag.
__device__ __forceinline__ void stage_x16(__half* xs, int xs_stride, const __half* src,
                                          const int* row_ids, int n, int cols) {
    const int chunks = cols >> 3;  // 16-byte chunks per row; 4 per block
    for (int i = threadIdx.x; i < n * chunks; i += blockDim.x) {
        const int r = i / chunks, c = i - r * chunks;
        const uint4 v = *reinterpret_cast<const uint4*>(src + (int64_t)row_ids[r] * cols + 8 * c);
        *reinterpret_cast<uint4*>(xs + r * xs_stride + (c >> 2) * kXBlockHalves + 8 * (c & 3)) = v;
    }
}

// Zeroes the shared zero block (block index cols/32 of token row 0's
// layout; the row stride leaves room for it, see diag_stride).
__device__ __forceinline__ void zero_block_init(__half* xs, int cols) {
    if (threadIdx.x < kXBlockHalves / 8)
        *reinterpret_cast<uint4*>(xs + (cols >> 5) * kXBlockHalves + 8 * threadIdx.x) =
            make_uint4(0u, 0u, 0u, 0u);
}

// Row stride of the staged x: the row's blocks plus one (the zero block
// lives in that slot of row 0).
__device__ __forceinline__ int diag_stride(int cols) { return ((cols >> 5) + 1) * kXBlockHalves; }

}  // namespace gw
