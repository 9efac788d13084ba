// gw_kernels.cu — sm_100a kernels of the MoE expert hot path.
//
//   k_prep          activation staging: router input in the compute dtype and
//                   the f16 expert input (bf16 rows prescaled by a power of two
//                   so every bf16 value converts to f16 exactly)
//   k_router        bf16 router GEMV + bias (Metal/MoE/router.metal:18-34); the
//                   last CTA to finish runs the top-k selection and softmax of
//                   Router.select (Runtime/Router.swift:78-98) for every token
//                   and builds the expert -> token lists
//   k_group         the same grouping for a routing decision supplied by the
//                   caller (ExpertRunner.applyAssignments' assignment set)
//   k_gateup        grouped MXFP4 gate_up GEMV + bias + activation epilogue
//                   (expert.metal:46-102, :380-393), one expert per CTA row
//   k_down          grouped MXFP4 down GEMV + bias, scaled by the routing weight
//                   (expert.metal:107-116 folded into the epilogue)
//   k_combine       per-token sum of its k expert contributions in rank order
//   k_gemv          batched plain MXFP4 GEMV (dequant_gemv.metal:37-67)
//   k_dequant       bit-exact MXFP4 decode (Quant/MXFP4.swift:48-92)
//   k_fill          seeded synthetic bank bytes
//   k_residual      stream += delta and the rounded next-layer input
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "gw_device.cuh"
#include "gw_internal.h"

namespace gw {

namespace {

__device__ __forceinline__ float load_act(const void* p, int dtype, int64_t i) {
    if (dtype == kF16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
    if (dtype == kBF16) return bf16_bits_to_f32(reinterpret_cast<const uint16_t*>(p)[i]);
    return reinterpret_cast<const float*>(p)[i];
}

__device__ __forceinline__ float round_to(float v, int dtype) {
    if (dtype == kF16) return __half2float(__float2half_rn(v));
    if (dtype == kBF16) return __bfloat162float(__float2bfloat16_rn(v));
    return v;
}

__device__ __forceinline__ void store_act(void* p, int dtype, int64_t i, float v) {
    if (dtype == kF16) reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
    else if (dtype == kBF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
    else reinterpret_cast<float*>(p)[i] = v;
}

// ---------------------------------------------------------------------------
// k_prep: one CTA per token.
//   src_dtype == round_dtype: the input is already in the compute dtype.
//   src_dtype == kF32: the residual stream, rounded to round_dtype first (and
//   written to xr_out for the router).
// f16 values pass through unscaled.  bf16 values are multiplied by 2^p, p
// chosen from the row's largest magnitude so that it lands in [2^15, 2^16);
// every bf16 value within 2^-24 of the row maximum is then an exact f16, and
// the GEMV multiplies its fp32 result by xmul = 2^-p.
__global__ void k_prep(const void* __restrict__ src, int src_dtype, int round_dtype, int H,
                       void* __restrict__ xr_out, __half* __restrict__ x16,
                       float* __restrict__ xmul) {
    const int t = blockIdx.x;
    __shared__ float red[32];
    float m = 0.f;
    for (int h = threadIdx.x; h < H; h += blockDim.x) {
        const float v = round_to(load_act(src, src_dtype, (int64_t)t * H + h), round_dtype);
        m = fmaxf(m, fabsf(v));
    }
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        v = warp_max(v);
        if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    m = red[0];
    int p = 0;
    if (round_dtype == kBF16 && m > 0.f && isfinite(m)) {
        int ex;
        frexpf(m, &ex);  // m < 2^ex
        p = 16 - ex;
        p = p < -120 ? -120 : (p > 120 ? 120 : p);
    }
    for (int h = threadIdx.x; h < H; h += blockDim.x) {
        const int64_t i = (int64_t)t * H + h;
        const float v = round_to(load_act(src, src_dtype, i), round_dtype);
        if (xr_out) store_act(xr_out, round_dtype, i, v);
        x16[i] = __float2half_rn(ldexpf(v, p));
    }
    if (threadIdx.x == 0) xmul[t] = ldexpf(1.f, -p);
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
__device__ void select_topk_warp(const float* __restrict__ logits, int E, int k, int* ord,
                                 int32_t* experts, float* weights) {
    const int lane = threadIdx.x & 31;
    for (int p = lane; p < E; p += 32) ord[p] = p;
    __syncwarp();
    for (int pos = 0; pos < k; ++pos) {
        float bv = 0.f;
        int bp = 0x7fffffff;
        bool have = false;
        for (int p = pos + ((lane - pos) & 31); p < E; p += 32) {
            const float v = __ldcg(logits + ord[p]);
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
            sel[j] = __ldcg(logits + ord[j]);
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
    }
    w.lists[(int64_t)e * w.tcap + pos] = slot;
}

// ---------------------------------------------------------------------------
// k_router: grid (ceil(E/4), ceil(T/8)), 4 warps; warp w scores expert
// 4*blockIdx.x + w against up to 8 tokens.  Each CTA then counts itself done;
// the last one selects the top-k of every token and groups the slots.
__global__ void __launch_bounds__(128) k_router(LayerView L, MoeDims d, const void* __restrict__ xr,
                                                int x_dtype, int T, MoeWork w) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e = blockIdx.x * 4 + warp;
    const int t0 = blockIdx.y * kTokTile;
    const int t1 = min(T, t0 + kTokTile);
    if (e < d.E) {
        const uint4* wrow = reinterpret_cast<const uint4*>(L.router_w + (int64_t)e * d.H);
        const int nchunk = d.H >> 3;
        const float bias = L.router_b ? bf16_bits_to_f32(L.router_b[e]) : 0.f;
        for (int t = t0; t < t1; ++t) {
            const uint4* xrow = reinterpret_cast<const uint4*>(
                reinterpret_cast<const char*>(xr) + ((int64_t)t * d.H) * (x_dtype == kF32 ? 4 : 2));
            float acc = 0.f;
            for (int c = lane; c < nchunk; c += 32) {
                const uint4 wv = __ldg(wrow + c);
                const uint4 xv = __ldg(xrow + c);
                const uint32_t wr[4] = {wv.x, wv.y, wv.z, wv.w};
                const uint32_t xx[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float w0 = __uint_as_float(wr[q] << 16);
                    const float w1 = __uint_as_float(wr[q] & 0xffff0000u);
                    float x0, x1;
                    if (x_dtype == kBF16) {
                        x0 = __uint_as_float(xx[q] << 16);
                        x1 = __uint_as_float(xx[q] & 0xffff0000u);
                    } else {
                        const __half2 h = *reinterpret_cast<const __half2*>(&xx[q]);
                        x0 = __low2float(h);
                        x1 = __high2float(h);
                    }
                    acc = fmaf(w0, x0, acc);
                    acc = fmaf(w1, x1, acc);
                }
            }
            acc = warp_sum(acc);
            if (lane == 0) w.logits[(int64_t)t * d.E + e] = acc + bias;
        }
    }

    __shared__ int last;
    __shared__ int ord[4][kMaxExperts];
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned total = gridDim.x * gridDim.y;
        const unsigned prev = atomicAdd(w.done, 1u);
        last = (prev == total - 1);
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (int i = threadIdx.x; i < d.E; i += blockDim.x) w.counts[i] = 0;
    if (threadIdx.x == 0) { *w.nactive = 0; *w.done = 0u; }
    __syncthreads();
    for (int t = warp; t < T; t += 4) {
        select_topk_warp(w.logits + (int64_t)t * d.E, d.E, d.k, ord[warp],
                         w.experts + (int64_t)t * d.k, w.weights + (int64_t)t * d.k);
        if (lane < d.k) group_slot(d, w, __ldcg(w.experts + (int64_t)t * d.k + lane), t * d.k + lane);
    }
}

// k_group: one CTA; a caller-supplied routing [T][k] (copied into the
// workspace) is grouped by expert.  Expert ids outside [0, E) are skipped.
__global__ void __launch_bounds__(256) k_group(MoeDims d, const int32_t* __restrict__ experts_in,
                                               const float* __restrict__ weights_in, int T, MoeWork w) {
    for (int i = threadIdx.x; i < d.E; i += blockDim.x) w.counts[i] = 0;
    if (threadIdx.x == 0) *w.nactive = 0;
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
// Grouped expert GEMVs.  grid (min(E, T*k), ceil(tiles / 4)), 4 warps: CTA
// (a, y) takes the a-th active expert and its 16-row tiles 4y..4y+3, and
// walks that expert's token list in blocks of 8 tokens staged in shared
// memory (row stride cols + 32 halves keeps the 16-byte fragment loads
// conflict-free).  Weight bytes are read once per 8 tokens.

__device__ __forceinline__ int xs_stride_for(int cols) { return cols + 32; }

__device__ __forceinline__ void stage_tokens(__half* xs, int xs_stride, const __half* src_rows,
                                             const int* row_ids, int n, int cols) {
    const int chunks = cols >> 3;  // 16-byte chunks per row
    for (int i = threadIdx.x; i < kTokTile * chunks; i += blockDim.x) {
        const int r = i / chunks, c = i - r * chunks;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (r < n) v = *reinterpret_cast<const uint4*>(src_rows + (int64_t)row_ids[r] * cols + 8 * c);
        *reinterpret_cast<uint4*>(xs + r * xs_stride + 8 * c) = v;
    }
}

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

template <int kAct>
__global__ void __launch_bounds__(kGemvWarps * 32) k_gateup(LayerView L, MoeDims d, int T, MoeWork w) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __half* xs = reinterpret_cast<__half*>(smem_raw);
    __shared__ int rows[kTokTile];
    __shared__ int slots[kTokTile];
    __shared__ float xm[kTokTile];
    const int a = blockIdx.x;
    if (a >= *w.nactive) return;
    const int e = w.active[a];
    const int cnt = min(w.counts[e], w.tcap);
    const int* list = w.lists + (int64_t)e * w.tcap;
    const uint8_t* ex = L.base + (int64_t)(e / d.shard_count) * L.stride;
    const uint8_t* packed = ex + L.off[0];
    const uint8_t* scales = ex + L.off[1];
    const uint16_t* bias = reinterpret_cast<const uint16_t*>(ex + L.off[4]);
    const int H = d.H, F = d.F;
    const int xs_stride = xs_stride_for(H);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int tile = blockIdx.y * kGemvWarps + warp;
    const int ntiles = F >> 3;  // 8 output features (16 interleaved rows) per tile
    const int f = tile * 8 + g;
    const int rowA = 2 * f, rowB = rowA + 1;
    float bA = 0.f, bB = 0.f;
    if (tile < ntiles) { bA = bf16_bits_to_f32(bias[rowA]); bB = bf16_bits_to_f32(bias[rowB]); }

    for (int c0 = 0; c0 < cnt; c0 += kTokTile) {
        const int n = min(kTokTile, cnt - c0);
        __syncthreads();
        if (threadIdx.x < kTokTile) {
            const int s = threadIdx.x < n ? list[c0 + threadIdx.x] : 0;
            slots[threadIdx.x] = s;
            rows[threadIdx.x] = s / d.k;
            xm[threadIdx.x] = threadIdx.x < n ? w.xmul[s / d.k] : 0.f;
        }
        __syncthreads();
        stage_tokens(xs, xs_stride, w.x16, rows, n, H);
        __syncthreads();
        if (tile < ntiles) {
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            mxfp4_tile<6>(packed, scales, H, rowA, rowB, xs, xs_stride, acc);
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const int col = 2 * t + q;
                if (col < n) {
                    const float gate = acc[q] * xm[col] + bA;
                    const float up = acc[2 + q] * xm[col] + bB;
                    const float v = activate<kAct>(gate, up, d.limit, d.alpha);
                    w.act[(int64_t)slots[col] * F + f] = __float2half_rn(v);
                }
            }
        }
    }
}

__global__ void __launch_bounds__(kGemvWarps * 32) k_down(LayerView L, MoeDims d, int T, MoeWork w) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __half* xs = reinterpret_cast<__half*>(smem_raw);
    __shared__ int slots[kTokTile];
    __shared__ float wt[kTokTile];
    const int a = blockIdx.x;
    if (a >= *w.nactive) return;
    const int e = w.active[a];
    const int cnt = min(w.counts[e], w.tcap);
    const int* list = w.lists + (int64_t)e * w.tcap;
    const uint8_t* ex = L.base + (int64_t)(e / d.shard_count) * L.stride;
    const uint8_t* packed = ex + L.off[2];
    const uint8_t* scales = ex + L.off[3];
    const uint16_t* bias = reinterpret_cast<const uint16_t*>(ex + L.off[5]);
    const int H = d.H, F = d.F;
    const int xs_stride = xs_stride_for(F);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int tile = blockIdx.y * kGemvWarps + warp;
    const int ntiles = H >> 4;
    const int rowA = tile * 16 + g, rowB = rowA + 8;
    float bA = 0.f, bB = 0.f;
    if (tile < ntiles) { bA = bf16_bits_to_f32(bias[rowA]); bB = bf16_bits_to_f32(bias[rowB]); }

    for (int c0 = 0; c0 < cnt; c0 += kTokTile) {
        const int n = min(kTokTile, cnt - c0);
        __syncthreads();
        if (threadIdx.x < kTokTile) {
            const int s = threadIdx.x < n ? list[c0 + threadIdx.x] : 0;
            slots[threadIdx.x] = s;
            wt[threadIdx.x] = threadIdx.x < n ? w.weights[s] : 0.f;
        }
        __syncthreads();
        stage_tokens(xs, xs_stride, w.act, slots, n, F);
        __syncthreads();
        if (tile < ntiles) {
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            mxfp4_tile<6>(packed, scales, F, rowA, rowB, xs, xs_stride, acc);
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const int col = 2 * t + q;
                if (col < n) {
                    float* y = w.ybuf + (int64_t)slots[col] * H;
                    y[rowA] = (acc[q] + bA) * wt[col];
                    y[rowB] = (acc[2 + q] + bB) * wt[col];
                }
            }
        }
    }
}

// k_combine: out[t][h] (=|+=) sum over ranks j of ybuf[t*k+j][h], skipping
// slots whose expert this shard does not own.  grid (ceil(H/4/256), T).
__global__ void k_combine(MoeDims d, MoeWork w, float* __restrict__ out, int accumulate) {
    const int t = blockIdx.y;
    const int h4 = blockIdx.x * blockDim.x + threadIdx.x;
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
        float4 p = *o;
        p.x += s.x; p.y += s.y; p.z += s.z; p.w += s.w;
        *o = p;
    } else {
        *o = s;
    }
}

// ---------------------------------------------------------------------------
// k_gemv: batched plain GEMV, y = dequant(W) x * xmul + bias.
// grid (count, ceil(rows/16/4)), 4 warps, one 16-row tile per warp.
__global__ void __launch_bounds__(kGemvWarps * 32) k_gemv(
    const uint8_t* __restrict__ packed, int64_t packed_stride, const uint8_t* __restrict__ scales,
    int64_t scale_stride, const uint16_t* __restrict__ bias, int64_t bias_stride,
    const __half* __restrict__ x16, int64_t x_stride, const float* __restrict__ xmul,
    float* __restrict__ y, int64_t y_stride, int rows, int cols) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __half* xs = reinterpret_cast<__half*>(smem_raw);
    const int m = blockIdx.x;
    const int xs_stride = xs_stride_for(cols);
    const int row_id = (x_stride == 0) ? 0 : m;
    const int chunks = cols >> 3;
    const __half* xsrc = x16 + (int64_t)row_id * cols;
    for (int i = threadIdx.x; i < kTokTile * chunks; i += blockDim.x) {
        const int r = i / chunks, c = i - r * chunks;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (r == 0) v = *reinterpret_cast<const uint4*>(xsrc + 8 * c);
        *reinterpret_cast<uint4*>(xs + r * xs_stride + 8 * c) = v;
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int tile = blockIdx.y * kGemvWarps + warp;
    if (tile * 16 >= rows) return;
    int rowA = tile * 16 + g, rowB = rowA + 8;
    const bool okA = rowA < rows, okB = rowB < rows;
    // Rows past the end read a valid row (row 0) and are not stored.
    const int rA = okA ? rowA : 0, rB = okB ? rowB : 0;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    mxfp4_tile<6>(packed + m * packed_stride, scales + m * scale_stride, cols, rA, rB, xs,
                  xs_stride, acc);
    if (t == 0) {
        const float mul = xmul[row_id];
        const uint16_t* bm = bias ? bias + m * bias_stride : nullptr;
        float* ym = y + m * y_stride;
        if (okA) ym[rowA] = acc[0] * mul + (bm ? bf16_bits_to_f32(bm[rowA]) : 0.f);
        if (okB) ym[rowB] = acc[2] * mul + (bm ? bf16_bits_to_f32(bm[rowB]) : 0.f);
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
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        if (kind == kFillCodes) {
            dst[i] = (uint8_t)(mix64(key + (uint64_t)(i >> 3)) >> (8 * (i & 7)));
        } else if (kind == kFillScales) {
            dst[i] = (uint8_t)(118 + mix64(key + (uint64_t)i) % 7);
        } else if (kind == kFillZero) {
            dst[i] = 0;
        } else if ((i & 1) == 0) {  // bf16 ~N(0, 0.02), one value per 2 bytes
            const uint64_t j = (uint64_t)(i >> 1);
            const double u1 = ((double)(mix64(key + 2 * j) >> 11) + 0.5) * (1.0 / 9007199254740992.0);
            const double u2 = (double)(mix64(key + 2 * j + 1) >> 11) * (1.0 / 9007199254740992.0);
            const double z = sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2) * 0.02;
            const __nv_bfloat16 b = __double2bfloat16(z);
            const uint16_t bits = *reinterpret_cast<const uint16_t*>(&b);
            dst[i] = (uint8_t)(bits & 0xff);
            if (i + 1 < n) dst[i + 1] = (uint8_t)(bits >> 8);
        }
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

inline int ok_or_fail() { return cudaPeekAtLastError() == cudaSuccess ? 1 : -1; }

}  // namespace

size_t gemv_smem_bytes(int cols) { return (size_t)kTokTile * (cols + 32) * sizeof(__half); }

int configure_kernels() {
    const int max_smem = 200 * 1024;
    if (cudaFuncSetAttribute(k_gateup<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem) != cudaSuccess) return -1;
    if (cudaFuncSetAttribute(k_gateup<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem) != cudaSuccess) return -1;
    if (cudaFuncSetAttribute(k_down, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem) != cudaSuccess) return -1;
    if (cudaFuncSetAttribute(k_gemv, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem) != cudaSuccess) return -1;
    return 0;
}

int launch_prep(const void* src, int src_dtype, int round_dtype, int T, int H, void* xr_out,
                __half* x16, float* xmul, cudaStream_t s) {
    if (T <= 0) return 0;
    k_prep<<<T, 256, 0, s>>>(src, src_dtype, round_dtype, H, xr_out, x16, xmul);
    return ok_or_fail();
}

int launch_router(const LayerView& L, const MoeDims& d, const void* xr, int x_dtype, int T,
                  const MoeWork& w, cudaStream_t s) {
    dim3 grid((d.E + 3) / 4, (T + kTokTile - 1) / kTokTile);
    k_router<<<grid, 128, 0, s>>>(L, d, xr, x_dtype, T, w);
    return ok_or_fail();
}

int launch_group(const MoeDims& d, const int32_t* experts_in, const float* weights_in, int T,
                 const MoeWork& w, cudaStream_t s) {
    k_group<<<1, 256, 0, s>>>(d, experts_in, weights_in, T, w);
    return ok_or_fail();
}

int launch_gateup(const LayerView& L, const MoeDims& d, int T, const MoeWork& w,
                  cudaStream_t s) {
    const int maxa = min(d.E, T * d.k);
    const int tiles = d.F / 8;
    dim3 grid(maxa, (tiles + kGemvWarps - 1) / kGemvWarps);
    if (d.act == 0)
        k_gateup<0><<<grid, kGemvWarps * 32, gemv_smem_bytes(d.H), s>>>(L, d, T, w);
    else
        k_gateup<1><<<grid, kGemvWarps * 32, gemv_smem_bytes(d.H), s>>>(L, d, T, w);
    return ok_or_fail();
}

int launch_down(const LayerView& L, const MoeDims& d, int T, const MoeWork& w, cudaStream_t s) {
    const int maxa = min(d.E, T * d.k);
    const int tiles = d.H / 16;
    dim3 grid(maxa, (tiles + kGemvWarps - 1) / kGemvWarps);
    k_down<<<grid, kGemvWarps * 32, gemv_smem_bytes(d.F), s>>>(L, d, T, w);
    return ok_or_fail();
}

int launch_combine(const MoeDims& d, int T, const MoeWork& w, float* out, int accumulate,
                   cudaStream_t s) {
    dim3 grid((d.H / 4 + 255) / 256, T);
    k_combine<<<grid, 256, 0, s>>>(d, w, out, accumulate);
    return ok_or_fail();
}

int launch_gemv_batched(int count, const uint8_t* packed, int64_t packed_stride,
                        const uint8_t* scales, int64_t scale_stride, const uint16_t* bias,
                        int64_t bias_stride, const __half* x16, int64_t x_stride,
                        const float* xmul, float* y, int64_t y_stride, int rows, int cols,
                        cudaStream_t s) {
    const int tiles = (rows + 15) / 16;
    dim3 grid(count, (tiles + kGemvWarps - 1) / kGemvWarps);
    k_gemv<<<grid, kGemvWarps * 32, gemv_smem_bytes(cols), s>>>(
        packed, packed_stride, scales, scale_stride, bias, bias_stride, x16, x_stride, xmul, y,
        y_stride, rows, cols);
    return ok_or_fail();
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

int launch_widen(const void* x, int x_dtype, float* stream, int64_t n, cudaStream_t s) {
    if (n <= 0) return 0;
    int64_t blocks = (n + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    k_widen<<<(unsigned)blocks, 256, 0, s>>>(x, x_dtype, stream, n);
    return ok_or_fail();
}

}  // namespace gw
