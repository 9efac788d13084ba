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

// One warp's 16-row x 8-column (tokens) MXFP4 tile over the full K.
//
// Fragment mapping (m16n8k16, g = lane/4, t = lane%4):
//   A rows: MMA row g    <- weight row rowA, MMA row g+8 <- weight row rowB.
//   K: for each 32-column block the thread owns packed word t (columns
//      8t..8t+7 of the block); byte 0/1 feed the first k16 step's low/high
//      k-pairs, bytes 2/3 the second's.  B is loaded with the same column
//      permutation: x[token g][block*32 + 8t .. 8t+7] as one 16-byte smem load.
//   C: c0 = (rowA, token 2t), c1 = (rowA, token 2t+1),
//      c2 = (rowB, token 2t), c3 = (rowB, token 2t+1).
// `xs` is the token block in shared memory, row stride `xs_stride` halves.
template <int kUnroll>
__device__ __forceinline__ void mxfp4_tile(const uint8_t* __restrict__ packed,
                                           const uint8_t* __restrict__ scales, int cols,
                                           int rowA, int rowB, const __half* xs, int xs_stride,
                                           float (&acc)[4]) {
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int nblk = cols >> 5;
    const uint32_t* pA = reinterpret_cast<const uint32_t*>(packed + (size_t)rowA * (cols >> 1)) + t;
    const uint32_t* pB = reinterpret_cast<const uint32_t*>(packed + (size_t)rowB * (cols >> 1)) + t;
    const uint8_t* sA = scales + (size_t)rowA * nblk;
    const uint8_t* sB = scales + (size_t)rowB * nblk;
    const __half* xr = xs + g * xs_stride + 8 * t;
    const float zero[4] = {0.f, 0.f, 0.f, 0.f};

    int b = 0;
    for (; b + kUnroll <= nblk; b += kUnroll) {
        uint32_t wa[kUnroll], wb[kUnroll], ea[kUnroll], eb[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            wa[u] = ldg_u32(pA + 4 * (b + u));
            wb[u] = ldg_u32(pB + 4 * (b + u));
            ea[u] = ldg_u8(sA + b + u);
            eb[u] = ldg_u8(sB + b + u);
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const uint4 xv = *reinterpret_cast<const uint4*>(xr + 32 * (b + u));
            uint32_t a0, a1, a2, a3, q0, q1, q2, q3;
            e2m1x8_to_f16x8(wa[u], a0, a1, a2, a3);
            e2m1x8_to_f16x8(wb[u], q0, q1, q2, q3);
            float d[4];
            mma16816(d, a0, q0, a1, q1, xv.x, xv.y, zero);
            mma16816(d, a2, q2, a3, q3, xv.z, xv.w, d);
            const float fa = gemv_scale(ea[u]), fb = gemv_scale(eb[u]);
            acc[0] = fmaf(d[0], fa, acc[0]);
            acc[1] = fmaf(d[1], fa, acc[1]);
            acc[2] = fmaf(d[2], fb, acc[2]);
            acc[3] = fmaf(d[3], fb, acc[3]);
        }
    }
    for (; b < nblk; ++b) {
        const uint32_t wa = ldg_u32(pA + 4 * b), wb = ldg_u32(pB + 4 * b);
        const uint32_t ea = ldg_u8(sA + b), eb = ldg_u8(sB + b);
        const uint4 xv = *reinterpret_cast<const uint4*>(xr + 32 * b);
        uint32_t a0, a1, a2, a3, q0, q1, q2, q3;
        e2m1x8_to_f16x8(wa, a0, a1, a2, a3);
        e2m1x8_to_f16x8(wb, q0, q1, q2, q3);
        float d[4];
        mma16816(d, a0, q0, a1, q1, xv.x, xv.y, zero);
        mma16816(d, a2, q2, a3, q3, xv.z, xv.w, d);
        const float fa = gemv_scale(ea), fb = gemv_scale(eb);
        acc[0] = fmaf(d[0], fa, acc[0]);
        acc[1] = fmaf(d[1], fa, acc[1]);
        acc[2] = fmaf(d[2], fb, acc[2]);
        acc[3] = fmaf(d[3], fb, acc[3]);
    }
}

}  // namespace gw
