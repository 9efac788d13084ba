// gw_stream.cu — decode-time expert GEMVs with the weights streamed by bulk
// copies.
//
// Same arithmetic as k_gateup / k_down (gw_kernels.cu) — the block-diagonal
// mma.sync tile of gw_device.cuh, group by group — but the weights no
// longer come through per-thread loads.  One persistent CTA per SM works through a contiguous
// range of items (expert token chunk of <= 4, 256-row tile):
//   warp 16     producer: one cp.async.bulk per 16-row tile and 8-block
//               group (a contiguous 16 x w x 16-byte run of the tiled bank,
//               plus its scale bytes) into a 4-group shared ring, i.e. about
//               136 KB of weights in flight per SM, signalled by mbarrier
//               transaction counts;
//   warps 0-15  consumers: warp j owns tile j of the item and runs the tile
//               math on each group straight from shared memory; the item's
//               tokens are staged once per (expert, chunk) in the padded x
//               layout the tile expects.
// This is the reference's per-token expert GEMV pair (mxfp4_gemv_bias ->
// activation -> mxfp4_gemv_bias, Metal/MoE/expert.metal:46-102, 311-368, driven
// by ExpertRunner.applyAssignments, Runtime/ExpertRunner.swift:108-183) for
// all of an expert's decode tokens at once.  Every wait is bounded; a wait
// that runs out sets a status bit and the CTA winds down.
#include <cuda_fp16.h>
#include <stdint.h>

#include "gw_async.cuh"
#include "gw_device.cuh"
#include "gw_internal.h"

namespace gw {
namespace {

constexpr int kSTok = kChunk;            // tokens per item (one staged chunk)
constexpr int kSGroups = 4;              // weight ring depth, in 8-block groups
constexpr int kSTileRun = 16 * 8 * 16;   // one 16-row tile's blocks of a full group
constexpr int kSConsumers = 16;          // consumer warps = 16-row tiles per item
constexpr int kSGroupPk = kSConsumers * kSTileRun;  // 32 KB of MXFP4 blocks per group
constexpr int kSGroupSc = kSConsumers * 16 * 8;     // 2 KB of scale bytes per group
constexpr int kSRows = kSConsumers * 16; // rows per item
constexpr int kSThreads = (kSConsumers + 1) * 32;
constexpr int kSRingBytes = kSGroups * (kSGroupPk + kSGroupSc);

#ifdef GW_STREAM_TRACE
__device__ unsigned long long g_stream_trace[8];
#endif

struct StreamArgs {
    LayerView L;
    MoeDims d;
    MoeWork w;
    int M, K;
    int sec_packed, sec_scales, sec_bias;
    int mode;  // 0 gate_up clamped GLU, 1 gate_up SiLU, 2 down
};

struct StreamShared {
    uint64_t gfull[kSGroups], gempty[kSGroups];
    int abort;
    int nact, nitems, mt;
    int prefix[kMaxExperts + 1];  // token chunks before active expert a
    int expert[kMaxExperts];
    int count[kMaxExperts];
    int slots[kSTok], rows[kSTok];
    float xm[kSTok];
};

struct SItem {
    int e, m0, c0, n;
    int key;  // (active expert, chunk): the staged tokens are reusable while it holds
};

// Items are numbered chunk-major, tile fastest: it = j * mt + m.
__device__ __forceinline__ SItem sdecode(const StreamShared& sh, int it) {
    const int j = it / sh.mt, m = it - j * sh.mt;
    int lo = 0, hi = sh.nact;
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (sh.prefix[mid] <= j) lo = mid; else hi = mid;
    }
    SItem r;
    r.e = sh.expert[lo];
    r.m0 = m * kSRows;
    r.c0 = (j - sh.prefix[lo]) * kSTok;
    r.n = min(kSTok, sh.count[lo] - r.c0);
    r.key = j;
    return r;
}

// Producer warp: every group of every item of this CTA's range.
__device__ __forceinline__ void stream_producer(StreamShared& sh, const StreamArgs& a, char* ring, int it0,
                                                int it1) {
    const int lane = threadIdx.x & 31;
    const int nblk = a.K >> 5, ngrp = (nblk + 7) >> 3;
    unsigned* status = a.w.status;
    int gq = 0;
    for (int it = it0; it < it1; ++it) {
        const SItem item = sdecode(sh, it);
        const uint8_t* ex = a.L.base + (int64_t)(item.e / a.d.shard_count) * a.L.stride;
        const int64_t tile0 = item.m0 >> 4;
        const uint8_t* pk = ex + a.L.off[a.sec_packed] + tile0 * 16 * nblk * 16;
        const uint8_t* sc = ex + a.L.off[a.sec_scales] + tile0 * 16 * nblk;
        const int tiles = min(kSConsumers, (a.M - item.m0) >> 4);
        for (int grp = 0; grp < ngrp; ++grp, ++gq) {
            const int slot = gq % kSGroups;
#ifdef GW_STREAM_TRACE
            const long long tp0 = clock64();
#endif
            if (!warp_wait(&sh.abort, &sh.gempty[slot], ((gq / kSGroups) & 1) ^ 1, status, 1u)) return;
#ifdef GW_STREAM_TRACE
            if (lane == 0) atomicAdd(&g_stream_trace[3], (unsigned long long)(clock64() - tp0));
#endif
            const int w = min(8, nblk - 8 * grp);
            const uint32_t run = 16 * w * 16, srun = 16 * w;
            char* dpk = ring + slot * (kSGroupPk + kSGroupSc);
            char* dsc = dpk + kSGroupPk;
            if (lane == 0) bar_arrive_tx(&sh.gfull[slot], tiles * (run + srun));
            __syncwarp();
            if (lane < tiles) {
                bulk_g2s(dpk + lane * kSTileRun, pk + (int64_t)lane * 16 * nblk * 16 + grp * 128 * 16, run,
                         &sh.gfull[slot]);
                bulk_g2s(dsc + lane * 128, sc + (int64_t)lane * 16 * nblk + grp * 128, srun, &sh.gfull[slot]);
            }
        }
    }
}

// One item of one consumer warp (tile j of the item), kTok / kSets as the
// GEMV tile's modes.  Returns false when the CTA is winding down.
template <int kTok, int kSets>
__device__ __forceinline__ bool stream_item(StreamShared& sh, const StreamArgs& a, const char* ring,
                                            const __half* xs, int xs_stride, const SItem& item, int j,
                                            int& gq, float (&oa)[kSTok], float (&ob)[kSTok]) {
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2;
    const int nblk = a.K >> 5, ngrp = (nblk + 7) >> 3;
    const bool valid = item.m0 + 16 * j < a.M;
    const int rowA = a.mode == 2 ? g : 2 * g, rowB = a.mode == 2 ? g + 8 : 2 * g + 1;
    float accA[kTok * kSets], accB[kTok * kSets];
#pragma unroll
    for (int q = 0; q < kTok * kSets; ++q) accA[q] = accB[q] = 0.f;
    for (int grp = 0; grp < ngrp; ++grp, ++gq) {
        const int slot = gq % kSGroups;
#ifdef GW_STREAM_TRACE
        const long long tw0 = clock64();
#endif
        if (!warp_wait(&sh.abort, &sh.gfull[slot], (gq / kSGroups) & 1, a.w.status, 2u)) return false;
#ifdef GW_STREAM_TRACE
        const long long tw1 = clock64();
#endif
        if (valid) {
            const int w = min(8, nblk - 8 * grp);
            const char* gb = ring + slot * (kSGroupPk + kSGroupSc);
            const uint4* tp = reinterpret_cast<const uint4*>(gb + j * kSTileRun);
            const uint8_t* ts = reinterpret_cast<const uint8_t*>(gb + kSGroupPk + j * 128);
            mxfp4_group_diag<kTok, kSets>(tp + rowA * w, tp + rowB * w, ts + rowA * w, ts + rowB * w, 8 * grp,
                                          nblk, xs, xs_stride, item.n, accA, accB);
        }
        __syncwarp();
        if (lane == 0) bar_arrive(&sh.gempty[slot]);
#ifdef GW_STREAM_TRACE
        if (lane == 0 && j == 0) {
            atomicAdd(&g_stream_trace[0], (unsigned long long)(tw1 - tw0));
            atomicAdd(&g_stream_trace[1], (unsigned long long)(clock64() - tw1));
            atomicAdd(&g_stream_trace[2], 1ull);
        }
#endif
    }
    quad_sum_acc(accA, accB);
#pragma unroll
    for (int q = 0; q < kSTok; ++q) {
        oa[q] = q < kTok * kSets ? accA[q < kTok * kSets ? q : 0] : 0.f;
        ob[q] = q < kTok * kSets ? accB[q < kTok * kSets ? q : 0] : 0.f;
    }
    return true;
}

// Consumer warps 0-15.  Barrier 1 (512 threads) orders the token staging; its
// reduction form makes the wind-down decision common to all consumers.
template <int kMode>
__device__ __forceinline__ void stream_consumers(StreamShared& sh, const StreamArgs& a, const char* ring,
                                                 __half* xs, int it0, int it1) {
    constexpr int kN = kSConsumers * 32;
    const int tid = threadIdx.x, j = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int cols = a.K, xs_stride = diag_stride(cols);
    const int chunks = cols >> 3;  // 16-byte pieces per staged row
    int gq = 0, staged = -1;
    bool ok = true;
    for (int it = it0; it < it1; ++it) {
        const SItem item = sdecode(sh, it);
        if (item.key != staged) {
            // everyone is done with the previous tokens, and goes on only if all can
            if (group_any(!ok, 1, kN)) return;
            if (tid < kSTok) {
                const bool live = tid < item.n;
                const int s = live ? a.w.lists[(int64_t)item.e * a.w.tcap + item.c0 + tid] : 0;
                sh.slots[tid] = s;
                sh.rows[tid] = kMode == 2 ? s : s / a.d.k;
                sh.xm[tid] = !live ? 0.f : (kMode == 2 ? a.w.weights[s] : a.w.xmul[s / a.d.k]);
            }
            group_sync(1, kN);
            const __half* src = kMode == 2 ? a.w.act : a.w.x16;
            for (int i = tid; i < item.n * chunks; i += kN) {
                const int r = i / chunks, c = i - r * chunks;
                const uint4 v = *reinterpret_cast<const uint4*>(src + (int64_t)sh.rows[r] * cols + 8 * c);
                *reinterpret_cast<uint4*>(xs + r * xs_stride + (c >> 2) * kXBlockHalves + 8 * (c & 3)) = v;
            }
            group_sync(1, kN);
            staged = item.key;
        }
        if (!ok) continue;  // winding down: no more waits, only the staging barriers
        float oa[kSTok], ob[kSTok];
        if (item.n == 1) ok = stream_item<1, 1>(sh, a, ring, xs, xs_stride, item, j, gq, oa, ob);
        else if (item.n == 2) ok = stream_item<2, 1>(sh, a, ring, xs, xs_stride, item, j, gq, oa, ob);
        else ok = stream_item<2, 2>(sh, a, ring, xs, xs_stride, item, j, gq, oa, ob);
        const int tile = (item.m0 >> 4) + j;
        if (!ok || t != 0 || item.m0 + 16 * j >= a.M) continue;
        const uint8_t* ex = a.L.base + (int64_t)(item.e / a.d.shard_count) * a.L.stride;
        const uint16_t* bias = reinterpret_cast<const uint16_t*>(ex + a.L.off[a.sec_bias]);
        if (kMode == 2) {  // down: rows tile*16 + g, + 8, times the routing weight
            const int rA = tile * 16 + g, rB = rA + 8;
            const float bA = bf16_bits_to_f32(bias[rA]), bB = bf16_bits_to_f32(bias[rB]);
            for (int q = 0; q < item.n; ++q) {
                float* y = a.w.ybuf + (int64_t)sh.slots[q] * a.M;
                y[rA] = (oa[q] + bA) * sh.xm[q];
                y[rB] = (ob[q] + bB) * sh.xm[q];
            }
        } else {  // gate_up: feature tile*8 + g from rows 2f (gate) and 2f + 1 (up)
            const int f = tile * 8 + g;
            const float bA = bf16_bits_to_f32(bias[2 * f]), bB = bf16_bits_to_f32(bias[2 * f + 1]);
            for (int q = 0; q < item.n; ++q) {
                const float v = activate<kMode>(oa[q] * sh.xm[q] + bA, ob[q] * sh.xm[q] + bB, a.d.limit, a.d.alpha);
                a.w.act[(int64_t)sh.slots[q] * a.d.F + f] = __float2half_rn(v);
            }
        }
    }
}

template <int kMode>
__global__ void __launch_bounds__(kSThreads, 1) k_stream(StreamArgs a) {
    extern __shared__ unsigned char dyn_s[];
    __shared__ StreamShared sh;
    char* ring = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(dyn_s) + 127) & ~uintptr_t(127));
    __half* xs = reinterpret_cast<__half*>(ring + kSRingBytes);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int mt = (a.M + kSRows - 1) / kSRows;

    const int nact = min(*a.w.nactive, a.d.E);
    for (int i = tid; i < nact; i += blockDim.x) {
        const int e = a.w.active[i];
        const int cnt = min(a.w.counts[e], a.w.tcap);
        sh.expert[i] = e;
        sh.count[i] = cnt;
        sh.prefix[i + 1] = (cnt + kSTok - 1) / kSTok;
    }
    if (tid == 0) {
        sh.abort = 0;
        sh.nact = nact;
        sh.mt = mt;
        for (int i = 0; i < kSGroups; ++i) { bar_init(&sh.gfull[i], 1); bar_init(&sh.gempty[i], kSConsumers); }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    zero_block_init(xs, a.K);
    __syncthreads();
    if (warp == 0) {  // exclusive prefix over <= 256 chunk counts, 8 per lane
        int v[8], sum = 0;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const int i = lane * 8 + q;
            v[q] = i < nact ? sh.prefix[i + 1] : 0;
            sum += v[q];
        }
        int incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        int run = incl - sum;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const int i = lane * 8 + q;
            if (i < nact) sh.prefix[i] = run;
            run += v[q];
        }
        if (lane == 31) { sh.prefix[nact] = incl; sh.nitems = incl * mt; }
    }
    __syncthreads();
    // a contiguous range of items per CTA, so consecutive items share their tokens
    const int n = sh.nitems;
    const int it0 = (int)((int64_t)n * blockIdx.x / gridDim.x), it1 = (int)((int64_t)n * (blockIdx.x + 1) / gridDim.x);
    if (warp < kSConsumers) stream_consumers<kMode>(sh, a, ring, xs, it0, it1);
    else stream_producer(sh, a, ring, it0, it1);
    __syncthreads();
    if (*(volatile int*)&sh.abort) {  // let bulk copies still in flight land before exiting
        const long long t0 = clock64();
        while (clock64() - t0 < 2000000) {}
    }
}

size_t stream_smem_bytes(int cols) {
    return 128 + kSRingBytes + (size_t)kSTok * ((cols >> 5) + 1) * kXBlockHalves * 2;
}

}  // namespace

int configure_stream(int max_cols) {
    const int bytes = (int)stream_smem_bytes(max_cols);
    if (cudaFuncSetAttribute(k_stream<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) return -1;
    if (cudaFuncSetAttribute(k_stream<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) return -1;
    if (cudaFuncSetAttribute(k_stream<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) return -1;
    return 0;
}

bool stream_supported(const MoeDims& d, const MoeWork& w) {
    // tiled 16-row tiles of 8-block groups; staged x of up to kStreamMaxCols
    return w.status != nullptr && d.H <= kStreamMaxCols && d.F <= kStreamMaxCols && d.H % 64 == 0 &&
           d.F % 64 == 0;
}

int launch_stream(const LayerView& L, const MoeDims& d, const MoeWork& w, int which, int sms, cudaStream_t s) {
    StreamArgs a;
    a.L = L;
    a.d = d;
    a.w = w;
    if (which == 0) {
        a.M = 2 * d.F; a.K = d.H;
        a.sec_packed = 0; a.sec_scales = 1; a.sec_bias = 4;
        a.mode = d.act == 0 ? 0 : 1;
    } else {
        a.M = d.H; a.K = d.F;
        a.sec_packed = 2; a.sec_scales = 3; a.sec_bias = 5;
        a.mode = 2;
    }
    const size_t smem = stream_smem_bytes(a.K);
    const dim3 grid(sms), block(kSThreads);
    if (a.mode == 0) k_stream<0><<<grid, block, smem, s>>>(a);
    else if (a.mode == 1) k_stream<1><<<grid, block, smem, s>>>(a);
    else k_stream<2><<<grid, block, smem, s>>>(a);
    return cudaGetLastError() == cudaSuccess ? 1 : -1;
}

#ifdef GW_STREAM_TRACE
extern "C" __attribute__((visibility("default"))) int gw_stream_trace(unsigned long long* out, int reset) {
    if (cudaMemcpyFromSymbol(out, g_stream_trace, sizeof(g_stream_trace)) != cudaSuccess) return -1;
    if (reset) {
        static const unsigned long long zero[8] = {};
        if (cudaMemcpyToSymbol(g_stream_trace, zero, sizeof(zero)) != cudaSuccess) return -1;
    }
    return 0;
}
#endif

}  // namespace gw
