// gw_kernels.cu — sm_100a kernels of the MoE expert hot path.
//
//   k_router        bf16 router GEMV + bias (Metal/MoE/router.metal:18-34), one
//                   expert x 8 tokens per CTA; the last CTA of a token chunk
//                   runs the top-k selection and softmax of Router.select
//                   (Runtime/Router.swift:78-98) for its tokens and builds the
//                   expert -> token lists
//   k_router_mma    the same for bf16 batches of >= 128 tokens, logits on mma.sync
//   k_rmsnorm       post-attention RMSNorm into the router input
//                   (Runtime/TransformerLayer.swift:265-285, router.metal:41-60)
//   k_group         the same grouping for a routing decision supplied by the
//                   caller (ExpertRunner.applyAssignments' assignment set)
//   k_gateup        grouped MXFP4 gate_up GEMV + bias + activation epilogue
//                   (expert.metal:46-102, :380-393), one expert per CTA row
//   k_down          grouped MXFP4 down GEMV + bias, scaled by the routing weight
//                   (expert.metal:107-116 folded into the epilogue)
//   k_combine       per-token sum of its k expert contributions in rank order,
//                   optionally added to the residual stream, which is then
//                   rounded into the next layer's input
//   k_gemv          batched plain MXFP4 GEMV (dequant_gemv.metal:37-67)
//   k_dequant       bit-exact MXFP4 decode (Quant/MXFP4.swift:48-92)
//   k_fill          seeded synthetic bank bytes
//   k_residual      stream += delta and the rounded next-layer input
//   k_widen         stream = x
//   k_xprep         x -> f16 with a per-row power-of-two shift (GEMV inputs)
//   k_tile_layout   reference row-major <-> tiled bank layout of one matrix
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "gw_async.cuh"
#include "gw_device.cuh"
#include "gw_internal.h"

namespace gw {

namespace {

__device__ __forceinline__ float load_act(const void* p, int dtype, int64_t i) {
    if (dtype == kF16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
    if (dtype == kBF16) return bf16_bits_to_f32(reinterpret_cast<const uint16_t*>(p)[i]);
    return reinterpret_cast<const float*>(p)[i];
}

__device__ __forceinline__ void store_act(void* p, int dtype, int64_t i, float v) {
    if (dtype == kF16) reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
    else if (dtype == kBF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
    else reinterpret_cast<float*>(p)[i] = v;
}

// ---------------------------------------------------------------------------
// Top-k selection of Router.select for one token, by one warp.
//
// The reference runs a partial selection sort over an index array: for each
// position it keeps the first candidate (in current array order) whose logit
// is strictly greater than the best so far, then swaps it into place.  The
// winner of each pass is therefore the smallest array position holding the
// maximum logit among positions >= pos.  The warp finds it with a (value,
// position) argmax reduction and performs the same swap, so ties resolve
// exactly as in the reference (by current array order, which the swaps
// perturb — not simply by lowest expert id).  NaN logits are outside this
// contract (the reference's own result then depends on scan order).
// The token's E logits are first copied (coalesced) into the warp's shared
// scratch `lg`, so the passes read shared memory, not L2.
__device__ void select_topk_warp(const float* __restrict__ logits_g, int E, int k, int* ord, float* lg,
                                 int32_t* experts, float* weights) {
    const int lane = threadIdx.x & 31;
    for (int p = lane; p < E; p += 32) {
        ord[p] = p;
        lg[p] = __ldcg(logits_g + p);
    }
    __syncwarp();
    const float* logits = lg;
    for (int pos = 0; pos < k; ++pos) {
        float bv = 0.f;
        int bp = 0x7fffffff;
        bool have = false;
        for (int p = pos + ((lane - pos) & 31); p < E; p += 32) {
            const float v = logits[ord[p]];
            if (!have || v > bv) { bv = v; bp = p; have = true; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int op = __shfl_xor_sync(0xffffffffu, bp, o);
            const bool oh = __shfl_xor_sync(0xffffffffu, have, o);
            const bool better = oh && (!have || ov > bv || (ov == bv && op < bp));
            if (better) { bv = ov; bp = op; have = oh; }
        }
        if (lane == 0) {
            const int tmp = ord[pos];
            ord[pos] = ord[bp];
            ord[bp] = tmp;
        }
        __syncwarp();
    }
    if (lane == 0) {
        // softmax over the selected logits only, max-subtracted, summed in order
        float sel[kMaxTopK];
        float peak = 0.f;
        for (int j = 0; j < k; ++j) {
            sel[j] = logits[ord[j]];
            if (j == 0 || sel[j] > peak) peak = sel[j];
        }
        float total = 0.f;
        for (int j = 0; j < k; ++j) {
            sel[j] = expf(sel[j] - peak);
            total += sel[j];
        }
        for (int j = 0; j < k; ++j) {
            experts[j] = ord[j];
            weights[j] = sel[j] / total;
        }
    }
    __syncwarp();
}

// Adds one (token, rank) slot to its expert's list if this shard owns it.
__device__ __forceinline__ void group_slot(const MoeDims& d, const MoeWork& w, int e, int slot) {
    if (e < 0 || e >= d.E || (e % d.shard_count) != d.shard_rank) return;
    const int pos = atomicAdd(w.counts + e, 1);
    if (pos >= w.tcap) return;  // a malformed routing listing an expert twice for a token
    if (pos == 0) {
        const int a = atomicAdd(w.nactive, 1);
        w.active[a] = e;
    } else if (pos % kGemvPass == 0) {  // the expert's tokens need one more GEMV pass
        const int a = atomicAdd(w.nextra, 1);
        w.extra[a] = e | ((pos / kGemvPass) << 16);
    }
    w.lists[(int64_t)e * w.tcap + pos] = slot;
}

// ---------------------------------------------------------------------------
// Converts one 32-value block of token row t to f16 with the row's shift p
// (x16 = x * 2^p; see row_exponent_shift).  One warp, lane = value.
__device__ __forceinline__ void prep_block(const void* x, int x_dtype, int H, int t, int blk, int p,
                                           __half* x16) {
    const int64_t i = (int64_t)t * H + blk * 32 + (threadIdx.x & 31);
    if (x_dtype == kF16) x16[i] = reinterpret_cast<const __half*>(x)[i];
    else x16[i] = __float2half_rn(bf16_bits_to_f32(reinterpret_cast<const uint16_t*>(x)[i]) * pow2f(p));
}

constexpr int kRouterSegs = (kMaxGemvCols + 255) / 256;  // 256-value hidden segments (banks cap H)

// k_router: grid (E, ceil(T/8)), kRouterWarps warps (16 for a single token
// chunk, where the grid is only E CTAs; 4 otherwise — both measured best on
// B200); CTA (e, y) scores expert e against the chunk's (up to) 8 tokens,
// warp w taking the w-th 1/kRouterWarps of the hidden dimension, and the
// partial sums meet in a fixed order.  The CTA also converts its share of those
// tokens' x blocks for the expert GEMVs.  Each CTA then counts itself done on
// its token chunk's counter; the last CTA of a chunk selects the top-k of the
// chunk's tokens and adds their slots to the expert lists (whose counts the
// previous combine left at zero).
template <int kRouterWarps, int kEpc>
__global__ void __launch_bounds__(kRouterWarps * 32, kRouterWarps == 4 ? 6 : 1) k_router(LayerView L, MoeDims d, const void* __restrict__ xr,
                                                int x_dtype, int T, MoeWork w) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e0 = blockIdx.x * kEpc;
    const int t0 = blockIdx.y * kTokTile;
    const int t1 = min(T, t0 + kTokTile);
    // The hidden dimension is cut into fixed segments of 32 8-value chunks (one
    // chunk per lane), each summed by one warp's tree; the warps take the
    // (expert, segment) units of the CTA's kEpc experts in turn and the
    // segment sums meet in segment order, so a token's logits come out
    // bit-identical whatever the warp count or the experts per CTA (and so
    // whatever the batch it is routed in).
    const int nchunk = d.H >> 3;
    const int nseg = (nchunk + 31) >> 5;
    __shared__ float racc[kEpc][kRouterSegs][kTokTile], rmx[kRouterWarps][kTokTile];
    __shared__ int shift[kTokTile];
    float mx[kTokTile];
#pragma unroll
    for (int q = 0; q < kTokTile; ++q) mx[q] = 0.f;
    for (int u = warp; u < kEpc * nseg; u += kRouterWarps) {
        const int le = u / nseg, sg = u - le * nseg;
        const int e = e0 + le;
        if (e >= d.E) break;
        const uint4* wrow = reinterpret_cast<const uint4*>(L.router_w + (int64_t)e * d.H);
        const int c = sg * 32 + lane;
        float acc[kTokTile];
#pragma unroll
        for (int q = 0; q < kTokTile; ++q) acc[q] = 0.f;
        if (c < nchunk) {
            // every load of the segment first (they are independent), then the math
            const uint4 wv = __ldg(wrow + c);
            uint4 xs[kTokTile];
#pragma unroll
            for (int q = 0; q < kTokTile; ++q)
                xs[q] = t0 + q < t1 ? __ldg(reinterpret_cast<const uint4*>(static_cast<const char*>(xr) +
                                                                          (int64_t)(t0 + q) * d.H * 2) + c)
                                    : make_uint4(0u, 0u, 0u, 0u);
            const uint32_t wr[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
            for (int q = 0; q < kTokTile; ++q) {
                if (t0 + q >= t1) break;
                const uint32_t xx[4] = {xs[q].x, xs[q].y, xs[q].z, xs[q].w};
#pragma unroll
                for (int v = 0; v < 4; ++v) {
                    float x0, x1;
                    if (x_dtype == kBF16) {
                        x0 = __uint_as_float(xx[v] << 16);
                        x1 = __uint_as_float(xx[v] & 0xffff0000u);
                    } else {
                        const __half2 h = *reinterpret_cast<const __half2*>(&xx[v]);
                        x0 = __low2float(h);
                        x1 = __high2float(h);
                    }
                    mx[q] = fmaxf(mx[q], fmaxf(fabsf(x0), fabsf(x1)));
                    acc[q] = fmaf(__uint_as_float(wr[v] << 16), x0, acc[q]);
                    acc[q] = fmaf(__uint_as_float(wr[v] & 0xffff0000u), x1, acc[q]);
                }
            }
        }
#pragma unroll
        for (int q = 0; q < kTokTile; ++q) {
            const float v = warp_sum(acc[q]);
            if (lane == 0) racc[le][sg][q] = v;
        }
    }
#pragma unroll
    for (int q = 0; q < kTokTile; ++q) {
        const float m = warp_max(mx[q]);
        if (lane == 0) rmx[warp][q] = m;
    }
    __syncthreads();
    if ((int)threadIdx.x < kEpc * kTokTile) {
        const int le = threadIdx.x / kTokTile, q = threadIdx.x % kTokTile;
        const int e = e0 + le;
        if (e < d.E && t0 + q < t1) {
            const float bias = L.router_b ? bf16_bits_to_f32(L.router_b[e]) : 0.f;
            float v = racc[le][0][q];
            for (int j = 1; j < nseg; ++j) v += racc[le][j][q];
            w.logits[(int64_t)(t0 + q) * d.E + e] = v + bias;
        }
    }
    if (warp == 0 && lane < kTokTile && t0 + lane < t1) {
        const int q = lane;
        float m = rmx[0][q];
#pragma unroll
        for (int j = 1; j < kRouterWarps; ++j) m = fmaxf(m, rmx[j][q]);
        const int p = x_dtype == kBF16 ? row_exponent_shift(m) : 0;
        shift[q] = p;
        if (blockIdx.x == 0) w.xmul[t0 + q] = pow2f(-p);
    }
    __syncthreads();
    // this CTA's share of the chunk's x blocks
    const int nblk = d.H >> 5;
    for (int task = blockIdx.x * kRouterWarps + warp; task < (t1 - t0) * nblk; task += gridDim.x * kRouterWarps)
        prep_block(xr, x_dtype, d.H, t0 + task / nblk, task % nblk, shift[task / nblk], w.x16);

    __shared__ int last;
    __shared__ int ord[kRouterWarps][kMaxExperts];
    __shared__ float lgc[kRouterWarps][kMaxExperts];
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned prev = atomicAdd(w.done + blockIdx.y, 1u);
        last = (prev == gridDim.x - 1);
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    if (threadIdx.x == 0) w.done[blockIdx.y] = 0u;
    for (int t = t0 + warp; t < t1; t += kRouterWarps) {
        select_topk_warp(w.logits + (int64_t)t * d.E, d.E, d.k, ord[warp], lgc[warp],
                         w.experts + (int64_t)t * d.k, w.weights + (int64_t)t * d.k);
        if (lane < d.k) group_slot(d, w, __ldcg(w.experts + (int64_t)t * d.k + lane), t * d.k + lane);
    }
}

// k_rmsnorm: the post-attention RMSNorm ahead of the router,
// out[t][i] = f16((stream[t][i] * inv) * w[i]), inv = 1 / sqrt(sum_i stream[t][i]^2 / H + eps),
// as TransformerLayer.normalise (Runtime/TransformerLayer.swift:265-285) and
// the Metal `rmsnorm` (Metal/MoE/router.metal:41-60) compute it: fp32 squares
// and sums, a plain multiplicative bf16 weight, IEEE division and square
// root, f16 output rounded to nearest even.  The reference sums the squares
// in index order; this kernel sums them as a tree (per-thread runs, then the
// warps), so `inv` can differ in its last bit and an output by one f16 ulp.
// grid T, 256 threads; H a multiple of 4.
__global__ void __launch_bounds__(256) k_rmsnorm(const float* __restrict__ stream,
                                                 const uint16_t* __restrict__ weight, float eps, int H,
                                                 __half* __restrict__ out) {
    const float* row = stream + (int64_t)blockIdx.x * H;
    __half* orow = out + (int64_t)blockIdx.x * H;
    float ss = 0.f;
    for (int i = threadIdx.x * 4; i < H; i += blockDim.x * 4) {
        const float4 v = *reinterpret_cast<const float4*>(row + i);
        ss = __fadd_rn(ss, __fmul_rn(v.x, v.x));
        ss = __fadd_rn(ss, __fmul_rn(v.y, v.y));
        ss = __fadd_rn(ss, __fmul_rn(v.z, v.z));
        ss = __fadd_rn(ss, __fmul_rn(v.w, v.w));
    }
    ss = warp_sum(ss);
    __shared__ float part[8];
    __shared__ float inv;
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        float tot = 0.f;
        for (int j = 0; j < (int)(blockDim.x >> 5); ++j) tot = __fadd_rn(tot, part[j]);
        inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)H), eps)));
    }
    __syncthreads();
    const float r = inv;
    for (int i = threadIdx.x * 4; i < H; i += blockDim.x * 4) {
        const float4 v = *reinterpret_cast<const float4*>(row + i);
        const uint2 wb = *reinterpret_cast<const uint2*>(weight + i);
        const float w0 = __uint_as_float(wb.x << 16), w1 = __uint_as_float(wb.x & 0xffff0000u);
        const float w2 = __uint_as_float(wb.y << 16), w3 = __uint_as_float(wb.y & 0xffff0000u);
        __half2* o = reinterpret_cast<__half2*>(orow + i);
        o[0] = __halves2half2(__float2half_rn(__fmul_rn(__fmul_rn(v.x, r), w0)),
                              __float2half_rn(__fmul_rn(__fmul_rn(v.y, r), w1)));
        o[1] = __halves2half2(__float2half_rn(__fmul_rn(__fmul_rn(v.z, r), w2)),
                              __float2half_rn(__fmul_rn(__fmul_rn(v.w, r), w3)));
    }
}

// k_xprep: x row -> f16 with the row's shift (see row_exponent_shift);
// grid (rows), one CTA per row, row m at x + m * x_stride elements.
__global__ void k_xprep(const void* __restrict__ x, int64_t x_stride, int x_dtype, int cols,
                        __half* __restrict__ x16, float* __restrict__ xmul) {
    const int m = blockIdx.x;
    const void* xm = static_cast<const char*>(x) + (size_t)m * x_stride * 2;
    __shared__ float red[32];
    __shared__ int shift;
    float mval = 0.f;
    if (x_dtype == kBF16)
        for (int i = threadIdx.x; i < cols; i += blockDim.x)
            mval = fmaxf(mval, fabsf(bf16_bits_to_f32(reinterpret_cast<const uint16_t*>(xm)[i])));
    mval = warp_max(mval);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mval;
    __syncthreads();
    if (threadIdx.x == 0) {
        float v = 0.f;
        for (int i = 0; i < (int)(blockDim.x >> 5); ++i) v = fmaxf(v, red[i]);
        shift = x_dtype == kBF16 ? row_exponent_shift(v) : 0;
        xmul[m] = pow2f(-shift);
    }
    __syncthreads();
    const int nblk = cols >> 5;
    for (int blk = threadIdx.x >> 5; blk < nblk; blk += blockDim.x >> 5)
        prep_block(xm, x_dtype, cols, 0, blk, shift, x16 + (size_t)m * cols);
}

// k_router_mma: the router for large bf16 batches.  grid ceil(T/16), 4 warps.
// A CTA owns 16 tokens outright: their row maxima (the x16 shift), the
// logits of all E experts (E a multiple of 32, <= 256) as a small GEMM on
// mma.sync.m16n8k16 bf16 (exact products, fp32 sums; warp w takes experts
// [w E/4, (w+1) E/4)), their x16 rows, and their top-k + grouping — so no
// cross-CTA completion counting is needed and each x row is read by one CTA
// instead of E/4.  Same results as k_router up to fp32 summation order
// (Router.logits, Runtime/Router.swift:38-66; Router.select :78-98).
__global__ void __launch_bounds__(128) k_router_mma(LayerView L, MoeDims d, const uint16_t* __restrict__ x,
                                                    int T, MoeWork w) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, tq = lane & 3;
    const int t0 = blockIdx.x * 16;
    const int H = d.H, E = d.E;
    __shared__ int shift[16];
    __shared__ int ord[4][kMaxExperts];
    __shared__ float lgc[4][kMaxExperts];
    // row maxima of the CTA's tokens: warp w takes tokens 4w .. 4w+3
    for (int q = 0; q < 4; ++q) {
        const int t = t0 + warp * 4 + q;
        float m = 0.f;
        if (t < T) {
            const uint4* xr = reinterpret_cast<const uint4*>(x + (int64_t)t * H);
            for (int c = lane; c < (H >> 3); c += 32) {
                const uint4 v = __ldg(xr + c);
                const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    m = fmaxf(m, fmaxf(fabsf(__uint_as_float(u[j] << 16)),
                                       fabsf(__uint_as_float(u[j] & 0xffff0000u))));
            }
        }
        m = warp_max(m);
        if (lane == 0) {
            const int p = t < T ? row_exponent_shift(m) : 0;
            shift[warp * 4 + q] = p;
            if (t < T) w.xmul[t] = pow2f(-p);
        }
    }
    // logits
    const int per = E >> 2, ntile = per >> 3;  // experts per warp, n-tiles of 8
    float c[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) c[n][0] = c[n][1] = c[n][2] = c[n][3] = 0.f;
    const int ra = min(t0 + g, T - 1), rb = min(t0 + g + 8, T - 1);  // rows past T reuse a valid row
    const uint32_t* xa = reinterpret_cast<const uint32_t*>(x + (int64_t)ra * H);
    const uint32_t* xb = reinterpret_cast<const uint32_t*>(x + (int64_t)rb * H);
    const uint32_t* wbase = reinterpret_cast<const uint32_t*>(L.router_w) + (int64_t)(warp * per + g) * (H >> 1);
#pragma unroll 4
    for (int k0 = 0; k0 < H; k0 += 16) {
        const int kk = (k0 >> 1) + tq;  // u32 holding columns k0 + 2 tq, + 1
        const uint32_t a0 = __ldg(xa + kk), a1 = __ldg(xb + kk), a2 = __ldg(xa + kk + 4), a3 = __ldg(xb + kk + 4);
#pragma unroll
        for (int n = 0; n < 8; ++n) {
            if (n < ntile) {
                const uint32_t* wr = wbase + (int64_t)n * 8 * (H >> 1);
                const uint32_t b0 = __ldg(wr + kk), b1 = __ldg(wr + kk + 4);
                asm volatile(
                    "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
                    "{%8,%9}, {%0,%1,%2,%3};"
                    : "+f"(c[n][0]), "+f"(c[n][1]), "+f"(c[n][2]), "+f"(c[n][3])
                    : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
            }
        }
    }
#pragma unroll
    for (int n = 0; n < 8; ++n) {
        if (n >= ntile) break;
        const int e0 = warp * per + n * 8 + 2 * tq;
        const float bias0 = L.router_b ? bf16_bits_to_f32(L.router_b[e0]) : 0.f;
        const float bias1 = L.router_b ? bf16_bits_to_f32(L.router_b[e0 + 1]) : 0.f;
        if (t0 + g < T) {
            w.logits[(int64_t)(t0 + g) * E + e0] = c[n][0] + bias0;
            w.logits[(int64_t)(t0 + g) * E + e0 + 1] = c[n][1] + bias1;
        }
        if (t0 + g + 8 < T) {
            w.logits[(int64_t)(t0 + g + 8) * E + e0] = c[n][2] + bias0;
            w.logits[(int64_t)(t0 + g + 8) * E + e0 + 1] = c[n][3] + bias1;
        }
    }
    __syncthreads();
    // the tokens' f16 rows (x * 2^shift, exact), eight values per thread and step
    const int n8 = H >> 3;
#pragma unroll 4
    for (int i = threadIdx.x; i < 16 * n8; i += blockDim.x) {
        const int q = i / n8, c8 = i - q * n8, t = t0 + q;
        if (t >= T) continue;
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(x + (int64_t)t * H) + c8);
        const float m = pow2f(shift[q]);
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const __half2 h = __floats2half2_rn(__uint_as_float(u[j] << 16) * m,
                                                __uint_as_float(u[j] & 0xffff0000u) * m);
            o[j] = *reinterpret_cast<const uint32_t*>(&h);
        }
        reinterpret_cast<uint4*>(w.x16 + (int64_t)t * H)[c8] = make_uint4(o[0], o[1], o[2], o[3]);
    }
    // their top-k and grouping
    for (int q = warp; q < 16; q += 4) {
        const int t = t0 + q;
        if (t >= T) break;
        select_topk_warp(w.logits + (int64_t)t * E, E, d.k, ord[warp], lgc[warp], w.experts + (int64_t)t * d.k,
                         w.weights + (int64_t)t * d.k);
        if (lane < d.k) group_slot(d, w, __ldcg(w.experts + (int64_t)t * d.k + lane), t * d.k + lane);
    }
}

// k_group: one CTA; a caller-supplied routing [T][k] (copied into the
// workspace) is grouped by expert.  Expert ids outside [0, E) are skipped.
__global__ void __launch_bounds__(256) k_group(MoeDims d, const int32_t* __restrict__ experts_in,
                                               const float* __restrict__ weights_in, int T, MoeWork w) {
    for (int i = threadIdx.x; i < d.E; i += blockDim.x) w.counts[i] = 0;
    if (threadIdx.x == 0) *w.nactive = *w.nextra = 0;
    __syncthreads();
    const int n = T * d.k;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int e = experts_in[i];
        w.experts[i] = e;
        w.weights[i] = weights_in[i];
        group_slot(d, w, e, i);
    }
}

// ---------------------------------------------------------------------------
// Grouped expert GEMVs.  grid (min(E, T*k), ceil(tiles / tiles_per_cta)),
// 4 warps: CTA (a, y) takes the a-th active expert; each of its warps owns one
// 16-row tile and a 1/ksplit share of the K blocks (ksplit = 1, 2 or 4 warps
// per tile, chosen by the host so that few-expert launches still fill the
// GPU).  As soon as the expert is known every warp queues its weight tile for
// L2; the expert's tokens are then walked in pairs staged in shared memory,
// so the tile streams from HBM once and any further pass (an expert chosen by
// 3+ tokens) hits L2.

// Block range of split `sp` out of `ksplit` (multiples of the 8-block group).
__device__ __forceinline__ void split_range(int nblk, int ksplit, int sp, int& b0, int& b1) {
    const int groups = (nblk + 7) >> 3;
    const int per = (groups + ksplit - 1) / ksplit;
    b0 = min(nblk, sp * per * 8);
    b1 = min(nblk, (sp + 1) * per * 8);
}

// Runs one token chunk (n = 1..kChunk) of a bank tile (tiled layout: packed /
// scales point at the tile, rowA / rowB are tile rows) split over `ksplit` warps
// and calls emit(token, rowA total, rowB total) once per (row pair, token)
// on the split-0 warp.  Every thread of the CTA must call this (it
// synchronises when ksplit > 1).  kPrefetch: see mxfp4_tile_diag.
// L2 prefetch policy of the two expert GEMVs (see mxfp4_tile_diag's
// kPrefetch): whole K-range up front for gate_up, two groups ahead for down.
constexpr int kPrefetchGateup = 1, kPrefetchDown = 2;
template <int kPrefetch, class Emit>
__device__ __forceinline__ void run_tile(int n, bool valid, const uint8_t* packed,
                                         const uint8_t* scales, int cols, int rowA, int rowB,
                                         const __half* xs, int ksplit, Emit&& emit) {
    __shared__ float red[kGemvWarps][8][2 * kChunk];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int sp = warp % ksplit;
    int b0, b1;
    split_range(cols >> 5, ksplit, sp, b0, b1);
    float a[kChunk], b[kChunk];
#pragma unroll
    for (int j = 0; j < kChunk; ++j) a[j] = b[j] = 0.f;
    if (valid) {
        const int st = diag_stride(cols);
        if (n == 1) {
            float a1[1], bb1[1];
            mxfp4_tile_diag<1, 1, true, false>(packed, scales, cols, rowA, rowB, xs, st, 1, b0, b1, a1, bb1);
            a[0] = a1[0];
            b[0] = bb1[0];
        } else if (n == 2) {
            float a2[2], bb2[2];
            mxfp4_tile_diag<2, 1, true, kPrefetch>(packed, scales, cols, rowA, rowB, xs, st, 2, b0, b1, a2, bb2);
            a[0] = a2[0]; a[1] = a2[1];
            b[0] = bb2[0]; b[1] = bb2[1];
        } else {
            mxfp4_tile_diag<2, 2, true, kPrefetch>(packed, scales, cols, rowA, rowB, xs, st, n, b0, b1, a, b);
        }
    }
    if (ksplit > 1) {
        if (t == 0) {
#pragma unroll
            for (int j = 0; j < kChunk; ++j) {
                red[warp][g][j] = a[j];
                red[warp][g][kChunk + j] = b[j];
            }
        }
        __syncthreads();
        if (sp == 0 && t == 0) {
            for (int q = 1; q < ksplit; ++q) {
#pragma unroll
                for (int j = 0; j < kChunk; ++j) {
                    a[j] += red[warp + q][g][j];
                    b[j] += red[warp + q][g][kChunk + j];
                }
            }
        }
        __syncthreads();
    }
    if (valid && sp == 0 && t == 0) {
#pragma unroll
        for (int j = 0; j < kChunk; ++j)
            if (j < n) emit(j, a[j], b[j]);
    }
}

template <int kAct>
__global__ void __launch_bounds__(kGemvWarps * 32, 5) k_gateup(LayerView L, MoeDims d, const void* x,
                                                              int x_dtype, int T, MoeWork w,
                                                              int ksplit) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __half* xs = reinterpret_cast<__half*>(smem_raw);
    __shared__ int rows[kChunk];
    __shared__ int slots[kChunk];
    __shared__ float xm[kChunk];
    const int a = blockIdx.x;
    if (a >= *w.nactive) return;
    const int e = w.active[a];
    const uint8_t* ex = L.base + (int64_t)(e / d.shard_count) * L.stride;
    const uint8_t* packed = ex + L.off[0];
    const uint8_t* scales = ex + L.off[1];
    const uint16_t* bias = reinterpret_cast<const uint16_t*>(ex + L.off[4]);
    const int H = d.H, F = d.F;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2;
    const int tile = blockIdx.y * (kGemvWarps / ksplit) + warp / ksplit;
    const int ntiles = F >> 3;  // 8 output features (16 interleaved rows) per tile
    const bool valid = tile < ntiles;
    const int f = tile * 8 + g;
    const int rowA = valid ? 2 * f : 0, rowB = rowA + 1;
    zero_block_init(xs, H);
    const int cnt = min(w.counts[e], w.tcap);
    const int* list = w.lists + (int64_t)e * w.tcap;
    float bA = 0.f, bB = 0.f;
    if (valid) { bA = bf16_bits_to_f32(bias[rowA]); bB = bf16_bits_to_f32(bias[rowB]); }

    for (int c0 = 0; c0 < cnt;) {
        const int n = min(kChunk, cnt - c0);
        __syncthreads();
        if (threadIdx.x < kChunk) {
            const int s = threadIdx.x < n ? list[c0 + threadIdx.x] : 0;
            slots[threadIdx.x] = s;
            rows[threadIdx.x] = s / d.k;
            xm[threadIdx.x] = threadIdx.x < n ? w.xmul[s / d.k] : 0.f;
        }
        __syncthreads();
        stage_x16(xs, diag_stride(H), w.x16, rows, n, H);
        __syncthreads();
        run_tile<kPrefetchGateup>(n, valid, packed + (size_t)tile * 16 * (H >> 1), scales + (size_t)tile * 16 * (H >> 5),
                 H, 2 * g, 2 * g + 1, xs, ksplit,
                 [&](int col, float ga, float ub) {
                     const float v = activate<kAct>(ga * xm[col] + bA, ub * xm[col] + bB, d.limit, d.alpha);
                     w.act[(int64_t)slots[col] * F + f] = __float2half_rn(v);
                 });
        c0 += n;
    }
}

__global__ void __launch_bounds__(kGemvWarps * 32, 5) k_down(LayerView L, MoeDims d, int T, MoeWork w,
                                                            int ksplit) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __half* xs = reinterpret_cast<__half*>(smem_raw);
    __shared__ int slots[kChunk];
    __shared__ float wt[kChunk];
    const int a = blockIdx.x;
    if (a >= *w.nactive) return;
    const int e = w.active[a];
    const uint8_t* ex = L.base + (int64_t)(e / d.shard_count) * L.stride;
    const uint8_t* packed = ex + L.off[2];
    const uint8_t* scales = ex + L.off[3];
    const uint16_t* bias = reinterpret_cast<const uint16_t*>(ex + L.off[5]);
    const int H = d.H, F = d.F;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2;
    const int tile = blockIdx.y * (kGemvWarps / ksplit) + warp / ksplit;
    const int ntiles = H >> 4;
    const bool valid = tile < ntiles;
    const int rowA = valid ? tile * 16 + g : 0, rowB = rowA + 8;
    zero_block_init(xs, F);
    const int cnt = min(w.counts[e], w.tcap);
    const int* list = w.lists + (int64_t)e * w.tcap;
    float bA = 0.f, bB = 0.f;
    if (valid) { bA = bf16_bits_to_f32(bias[rowA]); bB = bf16_bits_to_f32(bias[rowB]); }

    for (int c0 = 0; c0 < cnt;) {
        const int n = min(kChunk, cnt - c0);
        __syncthreads();
        if (threadIdx.x < kChunk) {
            const int s = threadIdx.x < n ? list[c0 + threadIdx.x] : 0;
            slots[threadIdx.x] = s;
            wt[threadIdx.x] = threadIdx.x < n ? w.weights[s] : 0.f;
        }
        __syncthreads();
        stage_x16(xs, diag_stride(F), w.act, slots, n, F);
        __syncthreads();
        run_tile<kPrefetchDown>(n, valid, packed + (size_t)tile * 16 * (F >> 1), scales + (size_t)tile * 16 * (F >> 5),
                 F, g, g + 8, xs, ksplit,
                 [&](int col, float ya, float yb) {
                     float* y = w.ybuf + (int64_t)slots[col] * H;
                     y[rowA] = (ya + bA) * wt[col];
                     y[rowB] = (yb + bB) * wt[col];
                 });
        c0 += n;
    }
}

// k_combine: s = sum over ranks j of ybuf[t*k+j] (skipping slots whose expert
// this shard does not own); out (=|+=) s; if x_next, x_next = round(out) in
// x_dtype.  grid (ceil(H/4/256), T).
__global__ void k_combine(MoeDims d, MoeWork w, float* __restrict__ out, int accumulate,
                          void* __restrict__ x_next, int x_dtype) {
    const int t = blockIdx.y;
    const int h4 = blockIdx.x * blockDim.x + threadIdx.x;
    // the expert lists have been consumed: leave the counts at zero for the
    // next router launch
    if (blockIdx.x == 0 && blockIdx.y == 0) {
        for (int i = threadIdx.x; i < d.E; i += blockDim.x) w.counts[i] = 0;
        if (threadIdx.x == 0) *w.nactive = *w.nextra = 0;
    }
    if (h4 * 4 >= d.H) return;
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < d.k; ++j) {
        const int e = w.experts[t * d.k + j];
        if (e < 0 || e >= d.E || (e % d.shard_count) != d.shard_rank) continue;
        const float4 v = reinterpret_cast<const float4*>(w.ybuf + (int64_t)(t * d.k + j) * d.H)[h4];
        s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
    }
    float4* o = reinterpret_cast<float4*>(out + (int64_t)t * d.H) + h4;
    if (accumulate) {
        const float4 p = *o;
        s.x += p.x; s.y += p.y; s.z += p.z; s.w += p.w;
    }
    *o = s;
    if (x_next) {
        const int64_t i = (int64_t)t * d.H + 4 * h4;
        store_act(x_next, x_dtype, i, s.x);
        store_act(x_next, x_dtype, i + 1, s.y);
        store_act(x_next, x_dtype, i + 2, s.z);
        store_act(x_next, x_dtype, i + 3, s.w);
    }
}

// ---------------------------------------------------------------------------
// k_gemv: batched plain GEMV, y = dequant(W) x + bias.  grid (count,
// ceil(rows/16/4)), 4 warps, one 16-row tile per warp, the block-diagonal
// single-token tile; x (f16 or bf16) is staged with per-block scales.
__global__ void __launch_bounds__(kGemvWarps * 32, 6) k_gemv(
    const uint8_t* __restrict__ packed, int64_t packed_stride, const uint8_t* __restrict__ scales,
    int64_t scale_stride, const uint16_t* __restrict__ bias, int64_t bias_stride,
    const __half* __restrict__ x16, const float* __restrict__ xmul, int x_stride,
    float* __restrict__ y, int64_t y_stride, int rows, int cols) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __half* xs = reinterpret_cast<__half*>(smem_raw);
    const int m = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int tile = blockIdx.y * kGemvWarps + warp;
    const int rowA = tile * 16 + g, rowB = rowA + 8;
    const bool okA = rowA < rows, okB = rowB < rows;
    // Rows past the end read a valid row (row 0) and are not stored.
    const int rA = okA ? rowA : 0, rB = okB ? rowB : 0;
    const uint8_t* pm = packed + m * packed_stride;
    const int xrow = x_stride == 0 ? 0 : m;
    zero_block_init(xs, cols);
    stage_x16(xs, diag_stride(cols), x16, &xrow, 1, cols);
    __syncthreads();
    if (tile * 16 >= rows) return;
    float a[1], b[1];
    mxfp4_tile_diag<1, 1>(pm, scales + m * scale_stride, cols, rA, rB, xs, diag_stride(cols), 1, 0,
                          cols >> 5, a, b);
    if (t == 0) {
        const uint16_t* bm = bias ? bias + m * bias_stride : nullptr;
        const float mul = xmul[xrow];
        float* ym = y + m * y_stride;
        if (okA) ym[rowA] = a[0] * mul + (bm ? bf16_bits_to_f32(bm[rowA]) : 0.f);
        if (okB) ym[rowB] = b[0] * mul + (bm ? bf16_bits_to_f32(bm[rowB]) : 0.f);
    }
}

// k_dequant: one thread per packed byte; MXFP4.decodeBlock's exact rule.
__global__ void k_dequant(const uint8_t* __restrict__ packed, const uint8_t* __restrict__ scales,
                          int64_t nbytes, float* __restrict__ w) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nbytes) return;
    const uint32_t byte = packed[i];
    const float s = decode_scale_exact(scales[i >> 4]);
    uint32_t h2;
    asm("{\n\t.reg .b8 q;\n\tcvt.u8.u32 q, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, q;\n\t}" : "=r"(h2) : "r"(byte));
    const __half2 hv = *reinterpret_cast<const __half2*>(&h2);
    w[2 * i] = __low2float(hv) * s;
    w[2 * i + 1] = __high2float(hv) * s;
}

// k_fill: synthetic bank bytes from the counter hash (see mix64).
__global__ void k_fill(uint8_t* __restrict__ dst, int64_t n, uint64_t key, int kind) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t first = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (kind == kFillBf16Normal) {  // bf16 ~N(0, 0.02), one value per 2 bytes
        uint16_t* out = reinterpret_cast<uint16_t*>(dst);
        for (int64_t j = first; j < n / 2; j += stride) {
            const uint64_t u = (uint64_t)j;
            const double u1 = ((double)(mix64(key + 2 * u) >> 11) + 0.5) * (1.0 / 9007199254740992.0);
            const double u2 = (double)(mix64(key + 2 * u + 1) >> 11) * (1.0 / 9007199254740992.0);
            const double z = sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2) * 0.02;
            // double -> fp32 (nearest) -> bf16 (nearest even), mirrored on the host
            out[j] = __bfloat16_as_ushort(__float2bfloat16_rn((float)z));
        }
        return;
    }
    for (int64_t i = first; i < n; i += stride) {
        if (kind == kFillCodes)
            dst[i] = (uint8_t)(mix64(key + (uint64_t)(i >> 3)) >> (8 * (i & 7)));
        else if (kind == kFillScales)
            dst[i] = (uint8_t)(118 + mix64(key + (uint64_t)i) % 7);
        else
            dst[i] = 0;
    }
}

// k_tile_layout: reference row-major MXFP4 matrix <-> the bank's tiled layout
// (tile_layout_offset).  `unit` bytes per element (16 for packed blocks, 1 for
// scales); rows % 16 == 0.  to_tiled = 0 converts back.
__global__ void k_tile_layout(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int rows,
                              int nblk, int unit, int to_tiled) {
    const int64_t n = (int64_t)rows * nblk;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const int row = (int)(i / nblk), blk = (int)(i - (int64_t)row * nblk);
        const int64_t t = tile_layout_offset(row, blk, nblk);
        const int64_t a = to_tiled ? i : t, b = to_tiled ? t : i;
        if (unit == 16)
            reinterpret_cast<uint4*>(dst)[b] = reinterpret_cast<const uint4*>(src)[a];
        else
            dst[b] = src[a];
    }
}

// k_residual: stream += delta; x_out = round(stream) in x_dtype (if given).
__global__ void k_residual(float* __restrict__ stream, const float* __restrict__ delta,
                           void* __restrict__ x_out, int x_dtype, int64_t n) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const float v = stream[i] + (delta ? delta[i] : 0.f);
        stream[i] = v;
        if (x_out) store_act(x_out, x_dtype, i, v);
    }
}

// k_widen: stream = x as fp32.
__global__ void k_widen(const void* __restrict__ x, int x_dtype, float* __restrict__ stream,
                        int64_t n) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        stream[i] = load_act(x, x_dtype, i);
}

// k_wait_probe: one CTA waits on an mbarrier that nothing ever completes,
// through the same bounded wait the warp-specialised kernels use, with a
// short limit; the wait gives up, sets kStatusProbe in the status word and
// the kernel returns.  Lets the host check its timeout reporting without a
// GPU fault.
__global__ void k_wait_probe(unsigned* status, long long limit) {
    __shared__ uint64_t never;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        bar_init(&never, 1);
        abort_flag = 0;
    }
    __syncthreads();
    if (threadIdx.x == 0) (void)wait_slow(&abort_flag, &never, 0, status, kStatusProbe, limit);
    __syncthreads();
}

inline int ok_or_fail() { return cudaPeekAtLastError() == cudaSuccess ? 1 : -1; }

// Warps per tile: split K when the expert work alone cannot fill the GPU
// (batch-1 decode runs only top_k experts per layer).
int pick_ksplit(int tiles_total) {
    // Measured on B200 at batch 1 (GPT-OSS and Qwen3 shapes): the best split is
    // the largest that keeps the launch under ~3072 warps (~20 per SM) — more
    // warps only add partial-sum reductions and per-CTA x staging.
    int ks = 1;
    while (ks < kGemvWarps && tiles_total * ks * 2 < 3072) ks *= 2;
    return ks;
}

}  // namespace

// Dynamic shared bytes of the expert kernels for `cols`-wide inputs.
size_t gemv_smem_bytes(int cols, int max_tok) {
    const size_t diag = (size_t)(cols / 32 + 1) * kXBlockHalves * sizeof(__half);
    return (size_t)std::min(std::max(max_tok, 1), kChunk) * diag;
}

int configure_kernels() {
    const int max_smem = 64 * 1024;
    if (cudaFuncSetAttribute(k_gateup<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem) != cudaSuccess) return -1;
    if (cudaFuncSetAttribute(k_gateup<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem) != cudaSuccess) return -1;
    if (cudaFuncSetAttribute(k_down, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem) != cudaSuccess) return -1;
    if (cudaFuncSetAttribute(k_gemv, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem) != cudaSuccess) return -1;
    return 0;
}

int launch_router(const LayerView& L, const MoeDims& d, const void* x, int x_dtype, int T,
                  const MoeWork& w, cudaStream_t s) {
    if (x_dtype == kBF16 && T >= kRouterMmaMinTokens && d.E % 32 == 0 && d.E <= kMaxExperts) {
        k_router_mma<<<(T + 15) / 16, 128, 0, s>>>(L, d, static_cast<const uint16_t*>(x), T, w);
        return ok_or_fail();
    }
    dim3 grid(d.E, (T + kTokTile - 1) / kTokTile);
    // one expert per CTA (8 experts per CTA, reading each token chunk once,
    // measured 1.9x slower at batch 64: too few warps in flight)
    if (T <= kTokTile) k_router<16, 1><<<grid, 16 * 32, 0, s>>>(L, d, x, x_dtype, T, w);
    else k_router<4, 1><<<grid, 4 * 32, 0, s>>>(L, d, x, x_dtype, T, w);
    return ok_or_fail();
}

int launch_group(const MoeDims& d, const int32_t* experts_in, const float* weights_in, int T,
                 const MoeWork& w, cudaStream_t s) {
    k_group<<<1, 256, 0, s>>>(d, experts_in, weights_in, T, w);
    return ok_or_fail();
}

int launch_gateup(const LayerView& L, const MoeDims& d, const void* x, int x_dtype, int T,
                  const MoeWork& w, cudaStream_t s) {
    const int maxa = min(d.E, T * d.k);
    const int tiles = d.F / 8;
    const int ks = pick_ksplit(tiles * maxa);
    const int per = kGemvWarps / ks;
    dim3 grid(maxa, (tiles + per - 1) / per);
    const size_t sm = gemv_smem_bytes(d.H, T);
    if (d.act == 0)
        k_gateup<0><<<grid, kGemvWarps * 32, sm, s>>>(L, d, x, x_dtype, T, w, ks);
    else
        k_gateup<1><<<grid, kGemvWarps * 32, sm, s>>>(L, d, x, x_dtype, T, w, ks);
    return ok_or_fail();
}

int launch_down(const LayerView& L, const MoeDims& d, int T, const MoeWork& w, cudaStream_t s) {
    const int maxa = min(d.E, T * d.k);
    const int tiles = d.H / 16;
    const int ks = pick_ksplit(tiles * maxa);
    const int per = kGemvWarps / ks;
    dim3 grid(maxa, (tiles + per - 1) / per);
    k_down<<<grid, kGemvWarps * 32, gemv_smem_bytes(d.F, T), s>>>(L, d, T, w, ks);
    return ok_or_fail();
}

int launch_combine(const MoeDims& d, int T, const MoeWork& w, float* out, int accumulate,
                   void* x_next, int x_dtype, cudaStream_t s) {
    dim3 grid((d.H / 4 + 255) / 256, T);
    k_combine<<<grid, 256, 0, s>>>(d, w, out, accumulate, x_next, x_dtype);
    return ok_or_fail();
}

int launch_rmsnorm(const float* stream, const uint16_t* weight, float eps, int T, int H, __half* out,
                  cudaStream_t s) {
    k_rmsnorm<<<T, 256, 0, s>>>(stream, weight, eps, H, out);
    return ok_or_fail();
}

int launch_xprep(const void* x, int x_dtype, int T, int H, __half* x16, float* xmul,
                 cudaStream_t s) {
    k_xprep<<<T, 256, 0, s>>>(x, H, x_dtype, H, x16, xmul);
    return ok_or_fail();
}

int launch_gemv_batched(int count, const uint8_t* packed, int64_t packed_stride,
                        const uint8_t* scales, int64_t scale_stride, const uint16_t* bias,
                        int64_t bias_stride, const void* x, int64_t x_stride, int x_dtype,
                        __half* x16, float* xmul, float* y, int64_t y_stride, int rows, int cols,
                        cudaStream_t s) {
    const int nx = x_stride == 0 ? 1 : count;
    k_xprep<<<nx, 256, 0, s>>>(x, x_stride, x_dtype, cols, x16, xmul);
    if (cudaPeekAtLastError() != cudaSuccess) return -1;
    const int tiles = (rows + 15) / 16;
    dim3 grid(count, (tiles + kGemvWarps - 1) / kGemvWarps);
    k_gemv<<<grid, kGemvWarps * 32, gemv_smem_bytes(cols, 1), s>>>(
        packed, packed_stride, scales, scale_stride, bias, bias_stride, x16, xmul,
        x_stride == 0 ? 0 : 1, y, y_stride, rows, cols);
    return cudaPeekAtLastError() == cudaSuccess ? 2 : -1;
}

int launch_dequant(const uint8_t* packed, const uint8_t* scales, int rows, int cols, float* w,
                   cudaStream_t s) {
    const int64_t nbytes = (int64_t)rows * cols / 2;
    if (nbytes == 0) return 0;
    const int64_t blocks = (nbytes + 255) / 256;
    k_dequant<<<(unsigned)blocks, 256, 0, s>>>(packed, scales, nbytes, w);
    return ok_or_fail();
}

int launch_fill_bytes(uint8_t* dst, int64_t n, uint64_t key, int kind, cudaStream_t s) {
    if (n <= 0) return 0;
    int64_t blocks = (n + 255) / 256;
    if (blocks > 148 * 64) blocks = 148 * 64;
    k_fill<<<(unsigned)blocks, 256, 0, s>>>(dst, n, key, kind);
    return ok_or_fail();
}

int launch_residual_round(float* stream, const float* delta, void* x_out, int x_dtype,
                          int64_t n, cudaStream_t s) {
    if (n <= 0) return 0;
    int64_t blocks = (n + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    k_residual<<<(unsigned)blocks, 256, 0, s>>>(stream, delta, x_out, x_dtype, n);
    return ok_or_fail();
}

int launch_tile_layout(const uint8_t* src, uint8_t* dst, int rows, int cols, int scales,
                       int to_tiled, cudaStream_t s) {
    const int nblk = cols / 32;
    int64_t blocks = ((int64_t)rows * nblk + 255) / 256;
    if (blocks > 148 * 32) blocks = 148 * 32;
    k_tile_layout<<<(unsigned)blocks, 256, 0, s>>>(src, dst, rows, nblk, scales ? 1 : 16, to_tiled);
    return ok_or_fail();
}

int launch_wait_probe(unsigned* status, long long limit, cudaStream_t s) {
    k_wait_probe<<<1, 32, 0, s>>>(status, limit);
    return ok_or_fail();
}

int launch_widen(const void* x, int x_dtype, float* stream, int64_t n, cudaStream_t s) {
    if (n <= 0) return 0;
    int64_t blocks = (n + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    k_widen<<<(unsigned)blocks, 256, 0, s>>>(x, x_dtype, stream, n);
    return ok_or_fail();
}

}  // namespace gw
