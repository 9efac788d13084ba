// gw_int8.cu — the trunk's int8 affine projections (output head, attention
// q/k/v/o) on the tensor cores.
//
// Format (Install/Int8Affine.swift, Install/Installer.swift:315-345): codes
// [rows][cols] uint8, then one bf16 (scale, zero) pair per row and group of 64
// columns, [rows][cols/64][2]; weight = code * scale + zero.  The reference
// kernels (Metal/MoE/router.metal:65-141, int8_affine_gemv and
// int8_affine_gemv_bias_batched) compute, per row and group, dot = sum q*x and
// xsum = sum x in fp32 and accumulate scale*dot + zero*xsum; the batched one
// adds the bf16 bias and rounds to f16.
//
// Here a warp owns a 16-row tile (or a K-split share of one) and walks its
// groups with 128-bit streaming loads: lane (g, t) reads bytes 16t..16t+15 of
// the group in rows g and g + 8.  Each byte pair becomes an exact f16x2 with
// one byte permute (0x64 above each byte: 1024 + code) and one f16x2
// subtract, and four mma.sync.m16n8k16 (f16 x f16 -> fp32, exact products)
// give the 16 rows' group dots for 8 tokens (N); the fp32 epilogue of each
// group is scale * dot + zero * xsum with the tokens' group sums computed once
// per CTA into shared memory.  The K order inside a group is permuted the same
// way for A and B (lane t's bytes 16t + 4m .. + 3 feed MMA m), so every
// operand comes from one register load.  x is read straight from global
// memory (it is a few KB and stays in L1); up to 8 * kNB tokens share each
// weight load, more tokens take further passes over the warp's tile.
#include <cuda_fp16.h>
#include <stdint.h>

#include <algorithm>

#include "gw_internal.h"

namespace gw {
namespace {

constexpr int kI8Warps = 8;           // warps per CTA
constexpr int kI8Unroll = 8;          // groups in flight per warp
constexpr int kI8MaxTok = 32;         // tokens per pass (kNB = 4)

struct Int8Args {
    const uint8_t* codes;
    const uint16_t* meta;
    const uint16_t* bias;  // or nullptr
    const __half* x;       // [T][cols]
    void* y;               // [T][rows] fp32 or f16
    int T, rows, cols;
    int ksplit;
    int y_f16;
};

__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// bytes 0,1 (sel 0x4140) or 2,3 (sel 0x4342) of w -> f16x2 of the two codes
template <uint32_t kSel>
__device__ __forceinline__ uint32_t u8x2_to_f16x2(uint32_t w) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(w), "r"(0x64646464u), "n"(kSel));
    const __half2 h = __hsub2(*reinterpret_cast<const __half2*>(&r), __half2(__float2half_rn(1024.f),
                                                                            __float2half_rn(1024.f)));
    return *reinterpret_cast<const uint32_t*>(&h);
}

// d = A B (kZero) or d += A B
template <bool kZero>
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    if (kZero)
        asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
            "{%10, %10, %10, %10};"
            : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
    else
        asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
            "{%0, %1, %2, %3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float bf16f(uint16_t v) { return __uint_as_float((uint32_t)v << 16); }

// grid: ceil(tiles / (kI8Warps / ksplit)) CTAs of kI8Warps warps; warp w works
// on tile blockIdx.x * (kI8Warps / ksplit) + w / ksplit, split w % ksplit.
template <int kNB>
__global__ void __launch_bounds__(kI8Warps * 32, kNB == 1 ? 2 : 1) k_int8_gemv(Int8Args a) {
    extern __shared__ float i8_smem[];
    const int ng = a.cols >> 6;
    const int tc = min(a.T, 8 * kNB);           // tokens per pass
    float* xs = i8_smem;                         // [tc][ng] group sums of this pass's tokens
    float* red = xs + tc * ng;                   // [kI8Warps][16][tc] split partials
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int ks = a.ksplit, tpc = kI8Warps / ks;
    const int tile = blockIdx.x * tpc + warp / ks, sp = warp % ks;
    const int per = (ng + ks - 1) / ks, gb = min(ng, sp * per), ge = min(ng, gb + per);
    const int r0 = tile * 16 + g, r1 = r0 + 8;
    const bool v0 = r0 < a.rows, v1 = r1 < a.rows;
    const uint8_t* w0 = a.codes + (int64_t)r0 * a.cols + 16 * t;
    const uint8_t* w1 = a.codes + (int64_t)r1 * a.cols + 16 * t;
    const uint32_t* m0 = reinterpret_cast<const uint32_t*>(a.meta) + (int64_t)r0 * ng;
    const uint32_t* m1 = reinterpret_cast<const uint32_t*>(a.meta) + (int64_t)r1 * ng;

    for (int t0 = 0; t0 < a.T; t0 += tc) {
        const int n = min(tc, a.T - t0);
        __syncthreads();  // the previous pass's sums and partials are consumed
        // group sums of the pass's tokens (fp32, as the reference's xsum)
        for (int i = threadIdx.x; i < n * ng; i += blockDim.x) {
            const int tok = i / ng, grp = i % ng;
            const uint4* p = reinterpret_cast<const uint4*>(a.x + (int64_t)(t0 + tok) * a.cols + grp * 64);
            float s = 0.f;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const uint4 v = __ldg(p + q);
                const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const float2 f = __half22float2(h[u]);
                    s += f.x + f.y;
                }
            }
            xs[tok * ng + grp] = s;
        }
        __syncthreads();
        // B rows: token nb * 8 + g of the pass (zero when absent)
        const __half* xr[kNB];
        bool xv[kNB];
#pragma unroll
        for (int nb = 0; nb < kNB; ++nb) {
            xv[nb] = nb * 8 + g < n;
            xr[nb] = a.x + (int64_t)(t0 + (xv[nb] ? nb * 8 + g : 0)) * a.cols + 16 * t;
        }
        float acc[kNB][4];
#pragma unroll
        for (int nb = 0; nb < kNB; ++nb) acc[nb][0] = acc[nb][1] = acc[nb][2] = acc[nb][3] = 0.f;
        // the tokens 2t, 2t + 1 of each column block whose sums this lane uses
        for (int grp0 = gb; grp0 < ge; grp0 += kI8Unroll) {
            uint4 wa[kI8Unroll], wb[kI8Unroll];
            uint32_t ma[kI8Unroll], mb[kI8Unroll];
#pragma unroll
            for (int u = 0; u < kI8Unroll; ++u) {
                const int grp = grp0 + u;
                const bool in = grp < ge;
                wa[u] = (in && v0) ? ldg_stream(w0 + grp * 64) : make_uint4(0, 0, 0, 0);
                wb[u] = (in && v1) ? ldg_stream(w1 + grp * 64) : make_uint4(0, 0, 0, 0);
                ma[u] = (in && v0) ? __ldg(m0 + grp) : 0u;
                mb[u] = (in && v1) ? __ldg(m1 + grp) : 0u;
            }
#pragma unroll
            for (int u = 0; u < kI8Unroll; ++u) {
                const int grp = grp0 + u;
                if (grp >= ge) break;
                float d[kNB][4];
                const uint32_t* pa = reinterpret_cast<const uint32_t*>(&wa[u]);
                const uint32_t* pb = reinterpret_cast<const uint32_t*>(&wb[u]);
                uint4 xq[kNB][2];
#pragma unroll
                for (int nb = 0; nb < kNB; ++nb) {
                    const uint4* px = reinterpret_cast<const uint4*>(xr[nb] + grp * 64);
                    xq[nb][0] = xv[nb] ? __ldg(px) : make_uint4(0, 0, 0, 0);
                    xq[nb][1] = xv[nb] ? __ldg(px + 1) : make_uint4(0, 0, 0, 0);
                }
#pragma unroll
                for (int m = 0; m < 4; ++m) {
                    // MMA m: lane bytes 4m..4m+3 of rows g (a0, a2) and g + 8 (a1, a3)
                    const uint32_t a0 = u8x2_to_f16x2<0x4140>(pa[m]);
                    const uint32_t a2 = u8x2_to_f16x2<0x4342>(pa[m]);
                    const uint32_t a1 = u8x2_to_f16x2<0x4140>(pb[m]);
                    const uint32_t a3 = u8x2_to_f16x2<0x4342>(pb[m]);
#pragma unroll
                    for (int nb = 0; nb < kNB; ++nb) {
                        // x[16t + 4m .. + 3] of the column's token: one 8-byte half of xq
                        const uint32_t* xw = reinterpret_cast<const uint32_t*>(&xq[nb][m >> 1]);
                        const uint32_t b0 = xw[(m & 1) * 2], b1 = xw[(m & 1) * 2 + 1];
                        if (m == 0) mma16816<true>(d[nb], a0, a1, a2, a3, b0, b1);
                        else mma16816<false>(d[nb], a0, a1, a2, a3, b0, b1);
                    }
                }
                const float s0 = bf16f((uint16_t)(ma[u] & 0xFFFFu)), z0 = bf16f((uint16_t)(ma[u] >> 16));
                const float s1 = bf16f((uint16_t)(mb[u] & 0xFFFFu)), z1 = bf16f((uint16_t)(mb[u] >> 16));
#pragma unroll
                for (int nb = 0; nb < kNB; ++nb) {
                    const int ta = nb * 8 + 2 * t;  // this lane's columns: tokens ta, ta + 1
                    const float xa = ta < n ? xs[ta * ng + grp] : 0.f;
                    const float xb = ta + 1 < n ? xs[(ta + 1) * ng + grp] : 0.f;
                    acc[nb][0] += fmaf(s0, d[nb][0], z0 * xa);
                    acc[nb][1] += fmaf(s0, d[nb][1], z0 * xb);
                    acc[nb][2] += fmaf(s1, d[nb][2], z1 * xa);
                    acc[nb][3] += fmaf(s1, d[nb][3], z1 * xb);
                }
            }
        }
        // K-split partials -> shared; split 0 sums them in split order and writes
        if (ks > 1) {
            float* rw = red + warp * 16 * tc;
#pragma unroll
            for (int nb = 0; nb < kNB; ++nb) {
                const int ta = nb * 8 + 2 * t;
                if (ta < n) { rw[g * tc + ta] = acc[nb][0]; rw[(g + 8) * tc + ta] = acc[nb][2]; }
                if (ta + 1 < n) { rw[g * tc + ta + 1] = acc[nb][1]; rw[(g + 8) * tc + ta + 1] = acc[nb][3]; }
            }
            __syncthreads();
            if (sp == 0) {
                const float* base = red + (warp - sp) * 16 * tc;
#pragma unroll
                for (int nb = 0; nb < kNB; ++nb) {
                    const int ta = nb * 8 + 2 * t;
#pragma unroll
                    for (int c = 0; c < 2; ++c) {
                        if (ta + c >= n) continue;
                        float y0 = 0.f, y1 = 0.f;
                        for (int q = 0; q < ks; ++q) {
                            y0 += base[q * 16 * tc + g * tc + ta + c];
                            y1 += base[q * 16 * tc + (g + 8) * tc + ta + c];
                        }
                        acc[nb][c] = y0;
                        acc[nb][2 + c] = y1;
                    }
                }
            }
        }
        if (sp == 0) {
            const float b0 = (a.bias && v0) ? bf16f(a.bias[r0]) : 0.f;
            const float b1 = (a.bias && v1) ? bf16f(a.bias[r1]) : 0.f;
#pragma unroll
            for (int nb = 0; nb < kNB; ++nb) {
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    const int tok = nb * 8 + 2 * t + c;
                    if (tok >= n) continue;
                    const int64_t o = (int64_t)(t0 + tok) * a.rows;
                    const float y0 = acc[nb][c] + b0, y1 = acc[nb][2 + c] + b1;
                    if (a.y_f16) {
                        __half* y = static_cast<__half*>(a.y) + o;
                        if (v0) y[r0] = __float2half_rn(y0);
                        if (v1) y[r1] = __float2half_rn(y1);
                    } else {
                        float* y = static_cast<float*>(a.y) + o;
                        if (v0) y[r0] = y0;
                        if (v1) y[r1] = y1;
                    }
                }
            }
        }
    }
}

// dynamic shared memory of a launch: the pass's group sums, and the split
// partials when the K range is split
size_t int8_smem(int tc, int cols, int ksplit) {
    return (size_t)tc * (cols / 64) * 4 + (ksplit > 1 ? (size_t)kI8Warps * 16 * tc * 4 : 0);
}

}  // namespace

int configure_int8() {
    const int bytes = (int)int8_smem(kI8MaxTok, kMaxInt8Cols, 2);
    for (auto fn : {k_int8_gemv<1>, k_int8_gemv<2>, k_int8_gemv<4>})
        if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) return -1;
    return 0;
}

int launch_int8_gemv(const uint8_t* codes, const uint16_t* meta, const uint16_t* bias, const __half* x,
                     int T, int rows, int cols, void* y, int y_f16, cudaStream_t s) {
    if (cols % 64 || cols > kMaxInt8Cols || rows <= 0 || T <= 0) return -1;
    static int sms[16] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 16) return -1;
    if (!sms[dev] && cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return -1;
    Int8Args a{codes, meta, bias, x, y, T, rows, cols, 1, y_f16};
    const int tiles = (rows + 15) / 16;
    // K-split: the fewest warps per tile that still put ~16 warps on every SM
    while (a.ksplit < kI8Warps && (int64_t)tiles * a.ksplit < (int64_t)sms[dev] * 16 &&
           cols / 64 >= 8 * a.ksplit)
        a.ksplit *= 2;
    const int tpc = kI8Warps / a.ksplit;
    const dim3 grid((tiles + tpc - 1) / tpc);
    const int tc = T <= 8 ? T : T <= 16 ? T : std::min(T, kI8MaxTok);
    const size_t smem = int8_smem(tc, cols, a.ksplit);
    if (T <= 8) k_int8_gemv<1><<<grid, kI8Warps * 32, smem, s>>>(a);
    else if (T <= 16) k_int8_gemv<2><<<grid, kI8Warps * 32, smem, s>>>(a);
    else k_int8_gemv<4><<<grid, kI8Warps * 32, smem, s>>>(a);
    return cudaPeekAtLastError() == cudaSuccess ? 1 : -1;
}

}  // namespace gw
