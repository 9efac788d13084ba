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
// One persistent CTA per SM walks a static list of work items (expert, token
// chunk of <= 128, 128-row tile).  Warp roles:
//   warps 0-7   converters: cp.async the tile's MXFP4 blocks and scale bytes
//               into a raw ring 7 stages ahead, then widen each 128 x 64
//               stage to f16 (cvt.rn.f16x2.e2m1x2, times the block scale) in
//               the canonical K-major layout tcgen05 reads.
//   warps 8-11  token loaders: cp.async the chunk's f16 activation rows into
//               the same stage.
//   warp 16     MMA issuer: one thread, tcgen05.mma kind::f16 M=128 N=n K=16,
//               fp32 accumulators in TMEM (two 128-column buffers so the
//               epilogue of one item overlaps the main loop of the next).
//   warps 12-15 epilogue: tcgen05.ld the accumulators (one row per thread),
//               scale, bias, activation / routing weight, store.
// Every wait is bounded (2 s); a wait that runs out sets a bit in the
// workspace status word and makes the whole CTA wind down: it drains its
// copies, waits for its MMAs and frees its TMEM before returning.
//
// f16 operands are exact: x16 rows are the router's power-of-two-shifted
// activations, and each weight row is multiplied by 2^(128 - emax_row) with
// emax_row the row's largest biased E8M0 exponent (precomputed per bank row):
// the row's largest blocks then hold e2m1 x 2^1 (at most 12) and every block
// within 25 binades of them is exact in f16 (normal or subnormal); blocks
// further down, whose products are below 2^-25 of the row's largest, flush to
// zero.  The epilogue undoes both shifts in fp32.
#include <cuda_fp16.h>
#include <stdint.h>

#include "gw_device.cuh"
#include "gw_internal.h"

namespace gw {
namespace {

constexpr int kM = 128;                  // weight rows per tile (MMA M)
constexpr int kNMax = 128;               // token columns per chunk (MMA N max)
constexpr int kKS = 64;                  // columns per stage (two MXFP4 blocks)
constexpr int kStages = 5;               // operand ring the MMA reads
constexpr int kRaw = 8;                  // raw weight ring depth (stages in flight)
constexpr int kScaleSlots = 6;           // per-group scale ring
constexpr int kASlot = kM * kKS * 2;     // 16 KB of f16 weights per stage
constexpr int kBSlot = kNMax * kKS * 2;  // 16 KB of f16 tokens per stage
constexpr int kRawSlot = kM * kKS / 2;   // 4 KB of MXFP4 blocks per stage
constexpr int kScaleSlot = 2 * kM * 16;  // 16 bytes per converter thread per 8-block group
constexpr int kRingBytes = kStages * (kASlot + kBSlot);
constexpr int kRawOff = kRingBytes;
constexpr int kScaleOff = kRawOff + kRaw * kRawSlot;
constexpr int kDynSmem = kScaleOff + kScaleSlots * kScaleSlot + 1024;  // + alignment slack
constexpr int kThreads = 17 * 32;
constexpr int kTmemCols = 2 * kNMax;
constexpr long long kWaitCycles = 4000000000ll;  // ~2 s at the B200's clocks

// Per-role cycle counters, compiled in with -DGW_GROUPED_TRACE: lane 0 of
// the first warp of each role adds the cycles it spent in each phase to
// g_grouped_trace[slot] (summed over CTAs); read with gw_grouped_trace().
#ifdef GW_GROUPED_TRACE
__device__ unsigned long long g_grouped_trace[16];
__device__ unsigned long long g_grouped_trace_conv;
#define GT_START(v) const long long v = clock64()
#define GT_ADD(slot, v, lead) \
    do { if (lead) atomicAdd(&g_grouped_trace[slot], (unsigned long long)(clock64() - (v))); } while (0)
#define GT_COUNT(slot, lead) \
    do { if (lead) atomicAdd(&g_grouped_trace[slot], 1ull); } while (0)
#else
#define GT_START(v) \
    do { } while (0)
#define GT_ADD(slot, v, lead) \
    do { } while (0)
#define GT_COUNT(slot, lead) \
    do { } while (0)
#endif

struct GroupedArgs {
    LayerView L;
    MoeDims d;
    MoeWork w;
    int M, K;                 // rows and columns of the expert matrix
    int sec_packed, sec_scales, sec_bias;
    int rexp_off;             // row offset of this matrix in the row-exponent table
    const __half* bsrc;       // token rows (x16 for gate_up, act for down)
    int bdiv;                 // token row = slot / bdiv
    int mode;                 // 0 gate_up clamped GLU, 1 gate_up SiLU, 2 down
};

// ---- PTX wrappers ---------------------------------------------------------
__device__ __forceinline__ uint32_t saddr(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void bar_init(uint64_t* b, uint32_t n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(b)), "r"(n) : "memory");
}
// True once the phase with `parity` has completed.
__device__ __forceinline__ bool bar_try(uint64_t* b, uint32_t parity) {
    uint32_t ok;
#ifdef GW_TRACE_TEST_WAIT
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(saddr(b)), "r"(parity)
        : "memory");
#else
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(saddr(b)), "r"(parity)
        : "memory");
#endif
    return ok != 0;
}
__device__ __forceinline__ void bar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(b)) : "memory");
}
__device__ __forceinline__ void fence_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void cp16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp8(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(saddr(dst)), "l"(src) : "memory");
}
// Arrives on `b` once every cp.async this thread issued so far has landed
// (counts as one of the barrier's expected arrivals).
__device__ __forceinline__ void cp_arrive_noinc(uint64_t* b) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(saddr(b)) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
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
__device__ __forceinline__ void tc_mma(uint32_t tmem, uint64_t ad, uint64_t bd, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
        "l"(ad), "l"(bd), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Shared-memory matrix descriptor, K-major, no swizzle: core matrices of 8
// rows x 16 bytes; lbo = byte distance between the two K-adjacent core
// matrices of one MMA, sbo = byte distance between 8-row groups.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | ((uint64_t)1 << 46);
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

// All threads of one role group (the 128 epilogue threads) agree on a flag.
__device__ __forceinline__ bool group_any(bool v, int id, int n) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.or.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(id), "r"(n)
        : "memory");
    return r != 0;
}
__device__ __forceinline__ void group_sync(int id, int n) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
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
    uint64_t full[kStages], empty[kStages], tfull[2], tempty[2], fin;
    uint32_t tmem;
    int abort;
    int nact, nitems;
    int prefix[kMaxExperts + 1];  // token chunks before active expert a
    int expert[kMaxExperts];
    int count[kMaxExperts];
    int col_slot[kNMax];          // epilogue: slot of each token column
    float col_mul[kNMax];         // epilogue: xmul (gate_up) or routing weight (down)
#ifdef GW_GROUPED_TRACE
    long long tok_issued[kStages], conv_arrived[kStages];
#endif
};

struct Item {
    int e, m0, c0, n;
};

// Items are numbered tile-major (item = m * chunks + j): CTAs that run at
// the same time take different experts' token chunks, so no set of token rows
// is read by dozens of SMs at once.
__device__ __forceinline__ Item decode(const Shared& sh, int it, int mt) {
    const int chunks = sh.nitems / mt;
    const int m = it / chunks, j = it - m * chunks;
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
    return r;
}

// Bounded wait; false when the CTA is winding down (this wait ran out, or
// another role's did).
__device__ __noinline__ bool wait_slow(Shared& sh, uint64_t* b, uint32_t parity, unsigned* status,
                                       unsigned bit) {
    const long long t0 = clock64();
    volatile int* ab = &sh.abort;
    for (uint32_t i = 1;; ++i) {
        if (bar_try(b, parity)) return true;
        if ((i & 63) == 0) {
            if (*ab) return false;
            if (clock64() - t0 > kWaitCycles) {
                *ab = 1;
                if (status) atomicOr(status, bit);
                return false;
            }
        }
    }
}
__device__ __forceinline__ bool wait_on(Shared& sh, uint64_t* b, uint32_t parity, unsigned* status,
                                        unsigned bit) {
    return bar_try(b, parity) || wait_slow(sh, b, parity, status, bit);
}

// ---- roles ----------------------------------------------------------------

// Converters: thread c owns weight row m0 + (c & 127) and, of each stage's
// two 32-column blocks, block (c >> 7).  One lane per warp does the ring's
// barrier work for its warp.
__device__ __forceinline__ void role_convert(Shared& sh, const GroupedArgs& a, char* smem, int mt) {
    const int c = threadIdx.x;
    const int r = c & (kM - 1), h = c >> 7, lane = c & 31;
    const int lr = r & 15;  // m0 is a multiple of 128
    const int nblk = a.K >> 5, ks = a.K / kKS;
    const int stride_g = gridDim.x;
    unsigned* status = a.w.status;
    char* raw = smem + kRawOff + h * (kRawSlot / 2) + r * 16;
    char* scl = smem + kScaleOff + h * (kScaleSlot / 2) + r * 16;

    // issue cursor (kRaw - 1 stages ahead of the consume cursor)
    int it_i = blockIdx.x, s_i = 0, g_i = 0, gr_i = 0;
    bool valid_i = false;
    const uint8_t *pk_i = nullptr, *sc_i = nullptr;
    int emax_pending = 127;
    auto issue = [&]() {
        if (it_i < sh.nitems) {
            if (s_i == 0) {
                const Item item = decode(sh, it_i, mt);
                const int R = item.m0 + r;
                valid_i = R < a.M;
                const int64_t le = item.e / a.d.shard_count;
                const uint8_t* ex = a.L.base + le * a.L.stride;
                const int64_t tile_blocks = (int64_t)(R >> 4) * 16 * nblk;
                pk_i = ex + a.L.off[a.sec_packed] + tile_blocks * 16;
                sc_i = ex + a.L.off[a.sec_scales] + tile_blocks;
                emax_pending = valid_i ? (int)a.L.rowexp[le * a.L.rowexp_stride + a.rexp_off + R] : 127;
            }
            const int grp = s_i >> 2, w = min(8, nblk - 8 * grp);
#ifdef GW_TRACE_SKIP_RAW
            if (false) {
#else
            if (valid_i) {
#endif
                const int64_t blk = (int64_t)grp * 128 + lr * w + ((2 * s_i + h) & 7);
                cp16(raw + (g_i % kRaw) * kRawSlot, pk_i + blk * 16);
                if ((s_i & 3) == 0) {
                    const int64_t off = (int64_t)grp * 128 + ((lr * w) & ~7);
                    char* sd = scl + (gr_i % kScaleSlots) * kScaleSlot;
                    cp8(sd, sc_i + off);
                    cp8(sd + 8, sc_i + off + 8);
                }
            }
            if ((s_i & 3) == 0) ++gr_i;
            ++g_i;
            if (++s_i == ks) { s_i = 0; it_i += stride_g; }
        }
        cp_commit();
    };

    for (int i = 0; i < kRaw - 1; ++i) issue();

    int it_c = blockIdx.x, s_c = 0, g_c = 0, gr_c = 0, gslot = 0, sub = 0;
    int emax = 127;
    bool valid_c = false;
    while (it_c < sh.nitems) {
        [[maybe_unused]] const bool lead = c == 0;
        if (s_c == 0) {
            const Item item = decode(sh, it_c, mt);
            valid_c = item.m0 + r < a.M;
            emax = emax_pending;
        }
        if ((s_c & 3) == 0) {
            const int w = min(8, nblk - 8 * (s_c >> 2));
            sub = (lr * w) & 7;
            gslot = gr_c % kScaleSlots;
            ++gr_c;
        }
        GT_START(t0);
        issue();
        cp_wait<kRaw - 1>();
        GT_ADD(0, t0, lead);
        GT_START(t1);
        uint4 out[4];
#ifdef GW_TRACE_SKIP_CONVERT
        if (false) {
#else
        if (valid_c) {
#endif
            const uint4 q = *reinterpret_cast<const uint4*>(raw + (g_c % kRaw) * kRawSlot);
            const uint8_t sb = *(reinterpret_cast<const uint8_t*>(scl + gslot * kScaleSlot) + sub +
                                 ((2 * s_c + h) & 7));
            const uint32_t hs = block_scale_h2(sb, emax);
            const uint32_t wd[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                out[j].x = hmul2_bits(e2m1x2(wd[j] & 0xFF), hs);
                out[j].y = hmul2_bits(e2m1x2((wd[j] >> 8) & 0xFF), hs);
                out[j].z = hmul2_bits(e2m1x2((wd[j] >> 16) & 0xFF), hs);
                out[j].w = hmul2_bits(e2m1x2(wd[j] >> 24), hs);
            }
        }
        const int slot = g_c % kStages;
        GT_ADD(1, t1, lead);
        GT_START(t2);
        bool ok = true;
        if (lane == 0) ok = wait_on(sh, &sh.empty[slot], ((g_c / kStages) & 1) ^ 1, status, 1u);
        if (!__shfl_sync(0xffffffffu, ok, 0)) break;
        GT_ADD(2, t2, lead);
        GT_START(t3);
        if (valid_c) {
            char* A = smem + slot * (kASlot + kBSlot) + (r >> 3) * 1024 + (r & 7) * 16 + h * 512;
#pragma unroll
            for (int j = 0; j < 4; ++j) *reinterpret_cast<uint4*>(A + j * 128) = out[j];
            fence_async_smem();
        }
        __syncwarp();
#ifdef GW_GROUPED_TRACE
        if (lead) *(volatile long long*)&sh.conv_arrived[slot] = clock64();
#endif
        if (lane == 0) bar_arrive(&sh.full[slot]);
        GT_ADD(3, t3, lead);
        GT_COUNT(13, lead);
        ++g_c;
        if (++s_c == ks) { s_c = 0; it_c += stride_g; }
    }
    cp_wait_all();
}

// Token loaders: thread t copies 16-byte column chunk (t & 7) of chunk rows
// (t >> 3) + 16 q, q = 0..7.  Completion is signalled to the stage's full
// barrier by the copies themselves, so the loaders run ahead as far as the
// ring allows.
__device__ __forceinline__ void role_tokens(Shared& sh, const GroupedArgs& a, char* smem, int mt) {
    constexpr int kRows = kNMax / 16;
    const int t = threadIdx.x - 256;
    const int c = t & 7, rb = t >> 3;
    const int ks = a.K / kKS;
    unsigned* status = a.w.status;
    int rid[kRows], nrid[kRows];
    auto load_rows = [&](int it, int (&dst)[kRows]) {
        if (it >= sh.nitems) return;
        const Item item = decode(sh, it, mt);
        const int32_t* list = a.w.lists + (int64_t)item.e * a.w.tcap + item.c0;
#pragma unroll
        for (int q = 0; q < kRows; ++q) {
            const int row = rb + 16 * q;
            dst[q] = row < item.n ? __ldg(list + row) / a.bdiv : -1;
        }
    };
    load_rows(blockIdx.x, nrid);
    int it = blockIdx.x, s = 0, g = 0;
    while (it < sh.nitems) {
        if (s == 0) {
#pragma unroll
            for (int q = 0; q < kRows; ++q) rid[q] = nrid[q];
            load_rows(it + gridDim.x, nrid);  // next item's rows, landing during this one
        }
        const int slot = g % kStages;
        GT_START(t0);
        if (!wait_on(sh, &sh.empty[slot], ((g / kStages) & 1) ^ 1, status, 2u)) break;
        GT_ADD(4, t0, t == 0);
        GT_START(t1);
        char* B = smem + slot * (kASlot + kBSlot) + kASlot + c * 128;
        const __half* src = a.bsrc + s * kKS + c * 8;
#pragma unroll
        for (int q = 0; q < kRows; ++q) {
            const int row = rb + 16 * q;
#ifndef GW_TRACE_SKIP_TOKENS
            if (rid[q] >= 0) cp16(B + (row >> 3) * 1024 + (row & 7) * 16, src + (int64_t)rid[q] * a.K);
#endif
        }
        cp_arrive_noinc(&sh.full[slot]);
        GT_ADD(5, t1, t == 0);
#ifdef GW_GROUPED_TRACE
        if (t == 0) *(volatile long long*)&sh.tok_issued[slot] = clock64();
#endif
        ++g;
        if (++s == ks) { s = 0; it += gridDim.x; }
    }
    cp_wait_all();
}

// MMA issuer: one thread.
__device__ __forceinline__ void role_mma(Shared& sh, const GroupedArgs& a, char* smem, int mt) {
    const int ks = a.K / kKS;
    unsigned* status = a.w.status;
    const uint32_t base = saddr(smem);
    int it = blockIdx.x, g = 0, il = 0;
    bool ok = true;
    while (ok && it < sh.nitems) {
        const Item item = decode(sh, it, mt);
        const int n = max(16, (item.n + 15) & ~15);
        const uint32_t idesc = (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kM >> 4) << 24);
        const int b = il & 1;
        GT_START(t0);
        if (!wait_on(sh, &sh.tempty[b], ((il >> 1) & 1) ^ 1, status, 4u)) break;
        GT_ADD(7, t0, true);
        tc_after_sync();
        const uint32_t tmem = sh.tmem + b * kNMax;
        for (int s = 0; s < ks; ++s, ++g) {
            const int slot = g % kStages;
            GT_START(t1);
            if (!wait_on(sh, &sh.full[slot], (g / kStages) & 1, status, 8u)) { ok = false; break; }
            GT_ADD(6, t1, true);
#ifdef GW_GROUPED_TRACE
            {
                // time from the token loads' issue / the converters' arrival to full
                const long long now = clock64();
                atomicAdd(&g_grouped_trace[15], (unsigned long long)(now - *(volatile long long*)&sh.tok_issued[slot]));
                atomicAdd(&g_grouped_trace_conv, (unsigned long long)(now - *(volatile long long*)&sh.conv_arrived[slot]));
            }
#endif
            GT_START(t2);
            tc_after_sync();
            fence_async_smem();  // token rows landed through cp.async (generic proxy)
            const uint32_t A = base + slot * (kASlot + kBSlot), B = A + kASlot;
#pragma unroll
            for (int k = 0; k < kKS / 16; ++k)
#ifndef GW_TRACE_SKIP_MMA
                tc_mma(tmem, smem_desc(A + k * 256, 128, 1024), smem_desc(B + k * 256, 128, 1024), idesc,
                       (s | k) != 0);
#else
                ;
#endif
            tc_commit(&sh.empty[slot]);
            GT_ADD(8, t2, true);
#ifdef GW_TRACE_COMMIT_LATENCY
            {
                GT_START(t3);
                while (!bar_try(&sh.empty[slot], (g / kStages) & 1)) {}
                GT_ADD(15, t3, true);
            }
#endif
        }
        if (!ok) break;
        tc_commit(&sh.tfull[b]);
        ++il;
        it += gridDim.x;
    }
    // every MMA this thread issued has finished before TMEM is freed
    tc_commit(&sh.fin);
    const long long t0 = clock64();
    while (!bar_try(&sh.fin, 0)) {
        if (clock64() - t0 > kWaitCycles) {
            if (status) atomicOr(status, 16u);
            break;
        }
    }
}

template <int kMode>
__device__ __forceinline__ void role_epilogue(Shared& sh, const GroupedArgs& a, int mt) {
    const int t = threadIdx.x - 384;  // 0..127 = TMEM lane = tile row
    const int ew = t >> 5, lane = t & 31;
    unsigned* status = a.w.status;
    int it = blockIdx.x, il = 0;
    while (it < sh.nitems) {
        GT_START(t0);
        const Item item = decode(sh, it, mt);
        const int R = item.m0 + t;
        const bool valid = R < a.M;
        const int64_t le = item.e / a.d.shard_count;
        const uint8_t* ex = a.L.base + le * a.L.stride;
        const uint16_t* bias = reinterpret_cast<const uint16_t*>(ex + a.L.off[a.sec_bias]);
        const int emax = valid ? (int)a.L.rowexp[le * a.L.rowexp_stride + a.rexp_off + R] : 127;
        const float bv = valid ? bf16_bits_to_f32(bias[R]) : 0.f;
        const int p = emax - 128, p1 = p / 2;  // undoes the 2^(1 - emax) row shift
        const float rs1 = pow2f(p1), rs2 = pow2f(p - p1);
        // column metadata for the chunk
        const int32_t* list = a.w.lists + (int64_t)item.e * a.w.tcap + item.c0;
        static_assert(kNMax == 128, "one column per epilogue thread");
        const int cs = t < item.n ? __ldg(list + t) : 0;
        const float cm = t < item.n ? (kMode == 2 ? a.w.weights[cs] : a.w.xmul[cs / a.d.k]) : 0.f;
        group_sync(1, 128);
        sh.col_slot[t] = cs;
        sh.col_mul[t] = cm;
        group_sync(1, 128);
        const int b = il & 1;
        GT_ADD(11, t0, t == 0);
        GT_START(t1);
        const bool got = wait_on(sh, &sh.tfull[b], (il >> 1) & 1, status, 32u);
        if (group_any(!got, 2, 128)) break;
        GT_ADD(9, t1, t == 0);
        GT_START(t2);
        tc_after_sync();
        const uint32_t taddr = sh.tmem + b * kNMax + ((uint32_t)(ew * 32) << 16);
        float pbv = __shfl_xor_sync(0xffffffffu, bv, 1);
#ifdef GW_TRACE_SKIP_EPILOGUE
        for (int j0 = 0; j0 < 0; j0 += 16) {
#else
        for (int j0 = 0; j0 < item.n; j0 += 16) {
#endif
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
                        const float y = activate<kMode>(acc * xm + bv, partner * xm + pbv, a.d.limit,
                                                            a.d.alpha);
                        a.w.act[(int64_t)sh.col_slot[col] * a.d.F + (R >> 1)] = __float2half_rn(y);
                    }
                }
            }
        }
        tc_before_sync();
        bar_arrive(&sh.tempty[b]);
        GT_ADD(10, t2, t == 0);
        GT_COUNT(14, t == 0);
        ++il;
        it += gridDim.x;
    }
}

template <int kMode>
__global__ void __launch_bounds__(kThreads, 1) k_grouped(GroupedArgs a) {
    extern __shared__ unsigned char dyn_raw[];
    __shared__ Shared sh;
    char* smem = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(dyn_raw) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int mt = (a.M + kM - 1) / kM;
    GT_START(tk);

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
        for (int i = 0; i < kStages; ++i) { bar_init(&sh.full[i], 8 + 128); bar_init(&sh.empty[i], 1); }
        for (int i = 0; i < 2; ++i) { bar_init(&sh.tfull[i], 1); bar_init(&sh.tempty[i], 128); }
        bar_init(&sh.fin, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
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
        if (lane == 31) { sh.prefix[nact] = incl; sh.nitems = incl * mt; }
    }
    __syncthreads();
    if (sh.nitems <= (int)blockIdx.x) return;  // no work for this CTA (uniform)
    if (warp == 16) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(&sh.tmem)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_before_sync();
    __syncthreads();
    tc_after_sync();

    if (warp < 8) role_convert(sh, a, smem, mt);
    else if (warp < 12) role_tokens(sh, a, smem, mt);
    else if (warp < 16) role_epilogue<kMode>(sh, a, mt);
    else if (lane == 0) role_mma(sh, a, smem, mt);

    tc_before_sync();
    __syncthreads();
    tc_after_sync();
    GT_ADD(12, tk, tid == 0);
    if (warp == 16)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(sh.tmem), "r"(kTmemCols)
                     : "memory");
}

}  // namespace

int grouped_smem_bytes() { return kDynSmem; }

int configure_grouped() {
    if (cudaFuncSetAttribute(k_grouped<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, kDynSmem) != cudaSuccess)
        return -1;
    if (cudaFuncSetAttribute(k_grouped<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kDynSmem) != cudaSuccess)
        return -1;
    if (cudaFuncSetAttribute(k_grouped<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, kDynSmem) != cudaSuccess)
        return -1;
    return 0;
}

bool grouped_supported(const MoeDims& d, const MoeWork& w) {
    // rows of both matrices split in 128-row tiles; columns in 64-column
    // stages, at least one raw ring's worth per item
    return w.status != nullptr && d.H % kKS == 0 && d.F % kKS == 0 && d.H / kKS >= kRaw &&
           d.F / kKS >= kRaw;
}

int launch_grouped(const LayerView& L, const MoeDims& d, const MoeWork& w, int which, int sms,
                   cudaStream_t s) {
    GroupedArgs a;
    a.L = L;
    a.d = d;
    a.w = w;
    if (which == 0) {
        a.M = 2 * d.F; a.K = d.H;
        a.sec_packed = 0; a.sec_scales = 1; a.sec_bias = 4;
        a.rexp_off = 0;
        a.bsrc = w.x16; a.bdiv = d.k;
        a.mode = d.act == 0 ? 0 : 1;
    } else {
        a.M = d.H; a.K = d.F;
        a.sec_packed = 2; a.sec_scales = 3; a.sec_bias = 5;
        a.rexp_off = 2 * d.F;
        a.bsrc = w.act; a.bdiv = 1;
        a.mode = 2;
    }
    const dim3 grid(sms), block(kThreads);
    if (a.mode == 0) k_grouped<0><<<grid, block, kDynSmem, s>>>(a);
    else if (a.mode == 1) k_grouped<1><<<grid, block, kDynSmem, s>>>(a);
    else k_grouped<2><<<grid, block, kDynSmem, s>>>(a);
    return cudaGetLastError() == cudaSuccess ? 1 : -1;
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

int launch_rowexp(const uint8_t* scales, int rows, int cols, uint8_t* out, cudaStream_t s) {
    k_rowexp<<<(rows + 127) / 128, 128, 0, s>>>(scales, rows, cols >> 5, out);
    return cudaGetLastError() == cudaSuccess ? 1 : -1;
}

#ifdef GW_GROUPED_TRACE
extern "C" __attribute__((visibility("default"))) int gw_grouped_trace(unsigned long long* out, int reset) {
    if (cudaMemcpyFromSymbol(out, g_grouped_trace, sizeof(g_grouped_trace)) != cudaSuccess) return -1;
    unsigned long long conv = 0;
    if (cudaMemcpyFromSymbol(&conv, g_grouped_trace_conv, sizeof(conv)) != cudaSuccess) return -1;
    out[16] = conv;
    if (reset) {
        static const unsigned long long zero[16] = {};
        if (cudaMemcpyToSymbol(g_grouped_trace, zero, sizeof(zero)) != cudaSuccess) return -1;
    }
    return 0;
}
#endif

}  // namespace gw
