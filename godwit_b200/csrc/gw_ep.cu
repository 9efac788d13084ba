// gw_ep.cu — the device side of token-sliced expert parallelism: packing a
// rank's (token, slot) rows into fixed-capacity per-peer blocks for the
// all-to-all dispatch, and summing the returned expert outputs per token.
//
// The reference runs on one device and has no counterpart; the semantics
// follow the single-device MoE block: the owner of expert e is rank e % world
// (the bank's expert sharding), a token's k partial outputs are summed in
// slot order (the order of k_combine and of ExpertRunner's accumulate,
// Metal/MoE/expert.metal:107-116).
//
// Send layout: world blocks of C rows; row = H values of the compute dtype
// followed by four 16-bit words holding the slot's expert id (int32, -1 for
// an unused row) and its routing weight (fp32 bits).  Slot s = t * k + j goes
// to row dest * C + pos, pos = the number of earlier slots bound for the
// same rank; a block that would need more than C rows sets *overflow and its
// extra slots share the block's last row (the host checks the flag).
#include <cuda_fp16.h>
#include <stdint.h>

#include "gw_internal.h"

namespace gw {
namespace {

constexpr int kEpPlanThreads = 1024;

// One CTA: row index of every slot, and the metadata words of every row.
__global__ void __launch_bounds__(kEpPlanThreads) k_ep_plan(const int32_t* __restrict__ experts,
                                                            const float* __restrict__ weights, int nslots,
                                                            int world, int C, int H, uint16_t* __restrict__ send,
                                                            int32_t* __restrict__ idx, int32_t* __restrict__ overflow) {
    __shared__ int running[kMaxEpWorld];
    __shared__ int wsum[kMaxEpWorld][kEpPlanThreads / 32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t rs = H + 4;  // row stride in 16-bit words
    if (tid < world) running[tid] = 0;
    __syncthreads();
    for (int base = 0; base < nslots; base += kEpPlanThreads) {
        const int s = base + tid;
        const int e = s < nslots ? experts[s] : -1;
        const int d = e >= 0 ? e % world : -1;
        int pos = 0;
        for (int r = 0; r < world; ++r) {
            const unsigned m = __ballot_sync(0xffffffffu, d == r);
            if (lane == 0) wsum[r][warp] = __popc(m);
            if (d == r) pos = __popc(m & ((1u << lane) - 1u));
        }
        __syncthreads();
        if (d >= 0) {
            int before = running[d];
            for (int w = 0; w < warp; ++w) before += wsum[d][w];
            pos += before;
            if (pos >= C) {
                atomicOr(overflow, 1);
                pos = C - 1;
            }
            const int row = d * C + pos;
            idx[s] = row;
            uint16_t* meta = send + (int64_t)row * rs + H;
            const uint32_t wb = __float_as_uint(weights[s]);
            meta[0] = (uint16_t)(e & 0xFFFF);
            meta[1] = (uint16_t)((uint32_t)e >> 16);
            meta[2] = (uint16_t)(wb & 0xFFFF);
            meta[3] = (uint16_t)(wb >> 16);
        } else if (s < nslots) {
            idx[s] = -1;
        }
        __syncthreads();
        if (tid < world) {
            int tot = 0;
            for (int w = 0; w < kEpPlanThreads / 32; ++w) tot += wsum[tid][w];
            running[tid] += tot;
        }
        __syncthreads();
    }
    // rows no slot took: expert -1 (skipped by the owner's grouping)
    for (int i = tid; i < world * C; i += blockDim.x) {
        const int d = i / C, p = i % C;
        if (p >= min(running[d], C)) {
            uint16_t* meta = send + (int64_t)i * rs + H;
            meta[0] = meta[1] = 0xFFFFu;
            meta[2] = meta[3] = 0;
        }
    }
}

// send[idx[s]][0:H] = x[s / k]: one CTA per slot, 16-byte copies (H % 8 == 0;
// rows of H + 4 16-bit words are 8-byte aligned, so the copy goes in 8 bytes).
__global__ void __launch_bounds__(128) k_ep_pack(const uint16_t* __restrict__ x, const int32_t* __restrict__ idx,
                                                 int k, int H, uint16_t* __restrict__ send) {
    const int s = blockIdx.x;
    const int row = idx[s];
    if (row < 0) return;
    const uint2* src = reinterpret_cast<const uint2*>(x + (int64_t)(s / k) * H);
    uint2* dst = reinterpret_cast<uint2*>(send + (int64_t)row * (H + 4));
    for (int i = threadIdx.x; i < H / 4; i += blockDim.x) dst[i] = __ldg(src + i);
}

// out[t] = sum over j of back[idx[t*k + j]] in slot order (rows of H fp32).
// grid (ceil(H/4/128), T), 128 threads.
__global__ void __launch_bounds__(128) k_ep_combine(const float* __restrict__ back, const int32_t* __restrict__ idx,
                                                    int k, int H, float* __restrict__ out) {
    const int t = blockIdx.y;
    const int h4 = blockIdx.x * blockDim.x + threadIdx.x;
    if (h4 * 4 >= H) return;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < k; ++j) {
        const int row = idx[t * k + j];
        if (row < 0) continue;
        const float4 v = __ldg(reinterpret_cast<const float4*>(back + (int64_t)row * H) + h4);
        acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    reinterpret_cast<float4*>(out + (int64_t)t * H)[h4] = acc;
}

}  // namespace

int launch_ep_dispatch(const void* x, int T, int H, const int32_t* experts, const float* weights, int k, int world,
                       int C, void* send, int32_t* idx, int32_t* overflow, cudaStream_t s) {
    if (world < 1 || world > kMaxEpWorld || C < 1 || H % 8) return -1;
    const int nslots = T * k;
    uint16_t* sd = static_cast<uint16_t*>(send);
    k_ep_plan<<<1, kEpPlanThreads, 0, s>>>(experts, weights, nslots, world, C, H, sd, idx, overflow);
    if (nslots > 0) k_ep_pack<<<nslots, 128, 0, s>>>(static_cast<const uint16_t*>(x), idx, k, H, sd);
    return cudaPeekAtLastError() == cudaSuccess ? (nslots > 0 ? 2 : 1) : -1;
}

int launch_ep_combine(const float* back, const int32_t* idx, int T, int k, int H, float* out, cudaStream_t s) {
    if (T <= 0) return 0;
    if (H % 4) return -1;
    k_ep_combine<<<dim3((H / 4 + 127) / 128, T), 128, 0, s>>>(back, idx, k, H, out);
    return cudaPeekAtLastError() == cudaSuccess ? 1 : -1;
}

}  // namespace gw
