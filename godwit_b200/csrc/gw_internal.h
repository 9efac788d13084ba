// gw_internal.h — launch-level interface between the C-ABI (gw_api.cu) and
// the kernels (gw_kernels.cu).  Nothing here crosses the library boundary.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace gw {

constexpr int kMaxTopK = 16;
constexpr int kMaxExperts = 256;
constexpr int kTokTile = 8;       // tokens per router CTA
constexpr int kRouterMmaMinTokens = 128;  // bf16 batches from here on use k_router_mma
constexpr int kGemvWarps = 4;     // warps per GEMV CTA (k_gemv, k_gateup, k_down: one 16-row tile each)
constexpr int kChunk = 4;         // tokens per weight pass of a k_gateup / k_down tile
constexpr int kGemvPass = 8;      // tokens per pass of the expert GEMV over an expert's weights

// Element types of activation inputs.  F32 is internal: the residual stream
// that the stack forward rounds to the configured input type.
enum Dtype : int { kF16 = 0, kBF16 = 1, kF32 = 2 };

// One layer of the resident bank as the kernels see it.
struct LayerView {
    const uint8_t* base;       // local expert 0's stride
    int64_t stride;            // bytes per expert stride
    int64_t off[6];            // section offsets within a stride
    const uint16_t* router_w;  // bf16 [E][H]
    const uint16_t* router_b;  // bf16 [E] or nullptr
    const uint8_t* rowexp;     // [E_local][2F + H] largest E8M0 exponent per weight row
    int64_t rowexp_stride;     // bytes per local expert in rowexp (2F + H)
};

struct MoeDims {
    int H, F, E, k, act;
    float limit, alpha;
    int shard_rank, shard_count;
};

// Scratch the MoE forward uses between kernels, sized for `tcap` tokens.
struct MoeWork {
    int tcap;
    void* xr;          // [tcap][H]   next layer's input in the compute dtype (stack mode)
    __half* x16;       // [tcap][H]   expert input as f16 (bf16 rows scaled by 1/xmul)
    float* xmul;       // [tcap]       power-of-two scale undoing each row's conversion shift
    float* logits;     // [tcap][E]
    int32_t* experts;  // [tcap][k]
    float* weights;    // [tcap][k]
    int32_t* counts;   // [E]          tokens routed to each expert
    int32_t* active;   // [E]          experts with at least one token (any order)
    int32_t* nactive;  // [1]
    int32_t* nextra;   // [1]          entries of `extra` (the word after *nactive)
    int32_t* extra;    // [tcap*k/kGemvPass+1] expert | pass << 16 for each further
                       //              kGemvPass-token pass an expert's tokens need
    int32_t* lists;    // [E][tcap]    slot ids (t*k + j) per expert
    __half* act;       // [tcap*k][F]  activated gate_up output (f16, as the reference); slot
                       //              order on the GEMV path, expert order on the tensor-core path
    __half* xg;        // [tcap*k][H]  x16 rows gathered in expert order (tensor-core path)
    uint8_t* xq;       // [tcap*k][H]  MXFP8 (E4M3) token rows in expert order (block-scaled mode)
    uint32_t* xsf;     // [tcap*k][ceil(H/128)] their E8M0 scales, 4 blocks per word
    uint8_t* aq;       // [tcap*k][F]  MXFP8 activations in expert order (block-scaled mode)
    uint32_t* asf;     // [tcap*k][ceil(F/128)]
    float* ybuf;       // [tcap*k][H]  routing-weighted down output per slot
    unsigned* done;    // [tcap/8+1]   router completion counter per token chunk (self-resetting)
    unsigned* status;  // [1]          sticky error bits set by bounded waits (nullptr: none)
    unsigned* sched;   // [2]          expert GEMV work counter and finished-CTA count (self-resetting)
    int mma_min_avg;   // tensor-core expert path when T*k >= mma_min_avg * E (0: never)
    int block_scaled;  // tensor-core path as block-scaled MXFP4 x MXFP8 MMAs (activations quantised)
};

// Host-side launchers; each returns the number of kernels it launched (or -1
// on a launch error, left in cudaGetLastError()).
int launch_router(const LayerView& L, const MoeDims& d, const void* x, int x_dtype, int T,
                  const MoeWork& w, cudaStream_t s);
int launch_group(const MoeDims& d, const int32_t* experts_in, const float* weights_in, int T,
                 const MoeWork& w, cudaStream_t s);
// Small-batch expert GEMVs (gw_kernels.cu): one active expert per CTA row,
// each warp one 16-row tile loaded by its own lanes with an L2 prefetch of
// the tile; the GEMV path's choice for layers of at most kSmallBatchSlots
// (token, slot) pairs, where their low launch latency beats the persistent
// TMA-fed kernel.
constexpr int kSmallBatchSlots = 8;
int launch_gateup(const LayerView& L, const MoeDims& d, const void* x, int x_dtype, int T,
                  const MoeWork& w, cudaStream_t s);
int launch_down(const LayerView& L, const MoeDims& d, int T, const MoeWork& w, cudaStream_t s);
int launch_combine(const MoeDims& d, int T, const MoeWork& w, float* out, int accumulate,
                   void* x_next, int x_dtype, cudaStream_t s);
int launch_gemv_batched(int count, const uint8_t* packed, int64_t packed_stride,
                        const uint8_t* scales, int64_t scale_stride, const uint16_t* bias,
                        int64_t bias_stride, const void* x, int64_t x_stride, int x_dtype,
                        __half* x16, float* xmul, float* y, int64_t y_stride, int rows, int cols,
                        cudaStream_t s);
int launch_dequant(const uint8_t* packed, const uint8_t* scales, int rows, int cols, float* w,
                   cudaStream_t s);
int launch_fill_bytes(uint8_t* dst, int64_t n, uint64_t key, int kind, cudaStream_t s);
int launch_residual_round(float* stream, const float* delta, void* x_out, int x_dtype,
                          int64_t n, cudaStream_t s);
int launch_xprep(const void* x, int x_dtype, int T, int H, __half* x16, float* xmul,
                 cudaStream_t s);
// out[T][H] f16 = RMSNorm(stream[T][H] fp32) with bf16 weight[H]; H % 4 == 0,
// 16-byte aligned rows.
int launch_rmsnorm(const float* stream, const uint16_t* weight, float eps, int T, int H, __half* out,
                   cudaStream_t s);
// Reference row-major <-> tiled bank layout of one MXFP4 matrix's packed
// blocks (scales = 0) or scale bytes (scales = 1).
int launch_tile_layout(const uint8_t* src, uint8_t* dst, int rows, int cols, int scales,
                       int to_tiled, cudaStream_t s);
// Status-word bit set by k_wait_probe (the kernels' own waits use bits 0-7).
constexpr unsigned kStatusProbe = 0x100u;
int launch_wait_probe(unsigned* status, long long limit, cudaStream_t s);
int launch_widen(const void* x, int x_dtype, float* stream, int64_t n, cudaStream_t s);
size_t gemv_smem_bytes(int cols, int max_tok);
// Tensor-core grouped expert GEMM (gw_grouped.cu): which 0 = gate_up + activation,
// 1 = down + routing weight.  `sms` persistent CTAs.
int launch_grouped(const LayerView& L, const MoeDims& d, const MoeWork& w, int which, int sms,
                   cudaStream_t s, const void* x = nullptr, int x_dtype = 0);
bool grouped_supported(const MoeDims& d, const MoeWork& w);
int configure_grouped();
// Decode expert GEMVs (gw_gemv.cu): which 0 = gate_up + activation, 1 =
// down + routing weight, for layers of T tokens on the GEMV path.
constexpr int kMaxGemvCols = 3072;  // the expert GEMV stages up to 12 groups of token blocks
int launch_expert_gemv(const LayerView& L, const MoeDims& d, const MoeWork& w, int T, int which,
                       cudaStream_t s);
bool expert_gemv_supported(const MoeDims& d);
int configure_expert_gemv();
// Trunk int8 affine GEMV (gw_int8.cu): y[T][rows] (fp32, or f16 when y_f16)
// = dequant(codes, meta) . x[t] (+ bf16 bias); cols % 64 == 0.
constexpr int kMaxInt8Cols = 16384;
int launch_int8_gemv(const uint8_t* codes, const uint16_t* meta, const uint16_t* bias, const __half* x,
                     int T, int rows, int cols, void* y, int y_f16, cudaStream_t s);
int configure_int8();
// Token-sliced expert parallelism (gw_ep.cu): pack (token, slot) rows into
// world blocks of C rows of H + 4 16-bit words; sum returned outputs per token.
constexpr int kMaxEpWorld = 64;
int launch_ep_dispatch(const void* x, int T, int H, const int32_t* experts, const float* weights, int k, int world,
                       int C, void* send, int32_t* idx, int32_t* overflow, cudaStream_t s);
int launch_ep_combine(const float* back, const int32_t* idx, int T, int k, int H, float* out, cudaStream_t s);
// Row-exponent table entries of a row-major scale matrix.
int launch_rowexp(const uint8_t* scales, int rows, int cols, uint8_t* out, cudaStream_t s);
int configure_kernels();

// Counter hash used by the synthetic bank generator (splitmix64 finaliser).
__host__ __device__ inline uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// Fill kinds for launch_fill_bytes.
enum FillKind : int { kFillCodes = 0, kFillScales = 1, kFillBf16Normal = 2, kFillZero = 3 };

}  // namespace gw
