/*
 * mxfp4_oracle.c — CPU restatement of rayl15/Godwit's MoE expert hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker and the timed
 * CPU baseline; it is never linked into, loaded by, or called from the
 * product library (godwit_b200/libgodwit_cuda.so).  Only tests/, the smoke
 * check in __graft_entry__.py and bench.py's CPU-baseline leg load it.
 *
 * Every function names the reference file:line whose arithmetic it restates
 * (paths inside rayl15/Godwit).  The reference is Swift + Metal and cannot be
 * compiled here, so this is a restatement in C with the same loop order and
 * fp32 arithmetic, not a compiled copy.  It is pinned against the reference's
 * own known-answer tests (Tests/GodwitTests/MXFP4Tests.swift,
 * MXFP4EncodeTests.swift, DequantGEMVTests.swift) and against golden vectors
 * produced by importing the reference's NumPy twin
 * (Scripts/analysis/expert_reference.py) — see tests/golden/make_golden.py.
 *
 * Values of x are passed as float arrays holding exactly the f16 / bf16
 * values the device sees; callers do the conversion.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define GWO_API __attribute__((visibility("default")))

/* MXFP4.codebook — Sources/Godwit/Quant/MXFP4.swift:22-25 */
static const float kCodebook[16] = {
    0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
    -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f,
};

/* MXFP4.thresholds — MXFP4.swift:106 (midpoints between magnitudes) */
static const float kThresholds[7] = {0.25f, 0.75f, 1.25f, 1.75f, 2.5f, 3.5f, 5.0f};

GWO_API float gwo_codebook(int code) { return kCodebook[code & 15]; }

/* MXFP4.decodeScale — MXFP4.swift:37-40: NaN for 0xFF, else 2^(byte-127). */
GWO_API float gwo_decode_scale(uint8_t byte) {
    if (byte == 0xFF) return NAN;
    return exp2f((float)((int)byte - 127));
}

/* MXFP4.decodeBlock / decode — MXFP4.swift:48-63, :69-92.
 * Low nibble holds the even-indexed weight. */
GWO_API void gwo_decode(const uint8_t* packed, const uint8_t* scales, int64_t block_count,
                        float* out) {
    for (int64_t b = 0; b < block_count; ++b) {
        const float scale = gwo_decode_scale(scales[b]);
        for (int i = 0; i < 16; ++i) {
            const uint8_t byte = packed[b * 16 + i];
            out[b * 32 + 2 * i] = kCodebook[byte & 0x0F] * scale;
            out[b * 32 + 2 * i + 1] = kCodebook[byte >> 4] * scale;
        }
    }
}

/* MXFP4.scaleByte(forPeak:) — MXFP4.swift:118-123: ceil(log2(peak/6)). */
GWO_API uint8_t gwo_scale_byte_for_peak(float peak) {
    if (!(peak > 0.0f) || !isfinite(peak)) return 127;
    const float exponent = ceilf(log2f(peak / 6.0f));
    int v = (int)exponent + 127;
    if (v == 255) v = 254;
    if (v < 0) v = 0;
    if (v > 255) v = 255;
    return (uint8_t)v;
}

/* MXFP4.code(forMagnitude:) — MXFP4.swift:127-134. */
GWO_API uint8_t gwo_code_for_magnitude(float value) {
    uint8_t code = 0;
    for (int i = 0; i < 7; ++i) {
        if (value < kThresholds[i]) return code;
        code += 1;
    }
    return code;
}

/* MXFP4.encodeBlock — MXFP4.swift:143-182; sign bit kept for values that
 * round to zero (code 8 = -0). `count` <= 32, short blocks zero-padded. */
static uint8_t encode_block(const float* w, int count, uint8_t* packed) {
    float peak = 0.0f;
    for (int i = 0; i < count; ++i)
        if (isfinite(w[i])) peak = fmaxf(peak, fabsf(w[i]));
    const uint8_t sb = gwo_scale_byte_for_peak(peak);
    const float inverse = 1.0f / gwo_decode_scale(sb);
    for (int j = 0; j < 16; ++j) {
        uint8_t byte = 0;
        for (int half = 0; half < 2; ++half) {
            const int idx = 2 * j + half;
            if (idx >= count) continue;
            const float v = w[idx];
            if (!isfinite(v)) continue;
            uint8_t nib = gwo_code_for_magnitude(fabsf(v) * inverse);
            if (signbit(v)) nib |= 0x08;
            byte |= half == 0 ? nib : (uint8_t)(nib << 4);
        }
        packed[j] = byte;
    }
    return sb;
}

/* MXFP4.encode — MXFP4.swift:188-207.  Returns the block count. */
GWO_API int64_t gwo_encode(const float* w, int64_t n, uint8_t* packed, uint8_t* scales) {
    const int64_t blocks = (n + 31) / 32;
    for (int64_t b = 0; b < blocks; ++b) {
        const int64_t start = b * 32;
        const int count = (int)((n - start) < 32 ? (n - start) : 32);
        scales[b] = encode_block(w + start, count, packed + b * 16);
    }
    return blocks;
}

/* DequantGEMVBenchmark.referenceMXFP4 — Benchmark/DequantGEMVBenchmark.swift:100-120,
 * same loop order: per block a 16-pair fp32 partial, then acc += partial*scale.
 * Plus the bf16 bias of mxfp4_gemv_bias (Metal/MoE/expert.metal:46-77);
 * `bias` may be NULL. */
static void gemv_rows(const uint8_t* packed, const uint8_t* scales, const float* bias,
                      const float* x, int64_t r0, int64_t r1, int64_t cols, float* y) {
    const int64_t bpr = cols / 32;
    for (int64_t row = r0; row < r1; ++row) {
        float acc = 0.0f;
        for (int64_t block = 0; block < bpr; ++block) {
            const float scale = gwo_decode_scale(scales[row * bpr + block]);
            const int64_t base = row * (cols / 2) + block * 16;
            const int64_t col0 = block * 32;
            float partial = 0.0f;
            for (int i = 0; i < 16; ++i) {
                const uint8_t byte = packed[base + i];
                partial += kCodebook[byte & 0x0F] * x[col0 + i * 2];
                partial += kCodebook[byte >> 4] * x[col0 + i * 2 + 1];
            }
            acc += partial * scale;
        }
        y[row] = bias ? acc + bias[row] : acc;
    }
}

GWO_API void gwo_gemv(const uint8_t* packed, const uint8_t* scales, const float* bias,
                      const float* x, int64_t rows, int64_t cols, float* y) {
    gemv_rows(packed, scales, bias, x, 0, rows, cols, y);
}

/* Same GEMV with rows split over `threads` POSIX threads (the all-cores CPU
 * baseline).  Results are identical to gwo_gemv: each row is one thread's. */
typedef struct {
    const uint8_t* packed; const uint8_t* scales; const float* bias; const float* x;
    int64_t r0, r1, cols; float* y;
} gemv_job;

static void* gemv_worker(void* p) {
    gemv_job* j = (gemv_job*)p;
    gemv_rows(j->packed, j->scales, j->bias, j->x, j->r0, j->r1, j->cols, j->y);
    return NULL;
}

GWO_API void gwo_gemv_mt(const uint8_t* packed, const uint8_t* scales, const float* bias,
                         const float* x, int64_t rows, int64_t cols, float* y, int threads) {
    if (threads <= 1) { gemv_rows(packed, scales, bias, x, 0, rows, cols, y); return; }
    if (threads > 256) threads = 256;
    pthread_t tid[256];
    gemv_job jobs[256];
    const int64_t per = (rows + threads - 1) / threads;
    int started = 0;
    for (int t = 0; t < threads; ++t) {
        const int64_t r0 = t * per, r1 = (t + 1) * per < rows ? (t + 1) * per : rows;
        if (r0 >= r1) break;
        jobs[t] = (gemv_job){packed, scales, bias, x, r0, r1, cols, y};
        if (pthread_create(&tid[t], NULL, gemv_worker, &jobs[t]) != 0) {
            gemv_worker(&jobs[t]);
            tid[t] = 0;
        }
        started = t + 1;
    }
    for (int t = 0; t < started; ++t)
        if (tid[t]) pthread_join(tid[t], NULL);
}

static inline float bf16_to_f32(uint16_t v) {
    uint32_t bits = (uint32_t)v << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static inline float round_f16(float v) { return (float)(_Float16)v; }

/* bf16_gemv_bias — Metal/MoE/router.metal:18-34: logits[e] = sum_c W[e,c]*x[c] + b[e],
 * fp32 accumulation (sequential here). `b` may be NULL (zeros). */
GWO_API void gwo_router_logits(const uint16_t* w, const uint16_t* b, const float* x,
                               int64_t E, int64_t H, float* logits) {
    for (int64_t e = 0; e < E; ++e) {
        float acc = 0.0f;
        for (int64_t c = 0; c < H; ++c) acc += bf16_to_f32(w[e * H + c]) * x[c];
        logits[e] = acc + (b ? bf16_to_f32(b[e]) : 0.0f);
    }
}

/* Router.select — Runtime/Router.swift:78-98: partial selection sort with a
 * strict '>' and swaps (ties resolve by current array order), then softmax
 * over the k selected logits only, max-subtracted. */
GWO_API void gwo_router_select(const float* logits, int E, int k, int32_t* experts,
                               float* weights) {
    int order[4096];
    for (int i = 0; i < E; ++i) order[i] = i;
    for (int pos = 0; pos < k; ++pos) {
        int best = pos;
        for (int cand = pos + 1; cand < E; ++cand)
            if (logits[order[cand]] > logits[order[best]]) best = cand;
        const int tmp = order[pos];
        order[pos] = order[best];
        order[best] = tmp;
    }
    float peak = -INFINITY;
    for (int j = 0; j < k; ++j) {
        experts[j] = order[j];
        if (j == 0 || logits[order[j]] > peak) peak = logits[order[j]];
    }
    float total = 0.0f;
    for (int j = 0; j < k; ++j) {
        weights[j] = expf(logits[order[j]] - peak);
        total += weights[j];
    }
    for (int j = 0; j < k; ++j) weights[j] = weights[j] / total;
}

/* gptoss_expert_activation — Metal/MoE/expert.metal:82-102: interleaved
 * gate/up, gate clamped above only, up clamped both ways, output rounded to
 * half.  Returned as float holding the half value. */
GWO_API void gwo_act_gptoss(const float* gate_up, int64_t F, float limit, float alpha,
                            float* out) {
    for (int64_t i = 0; i < F; ++i) {
        float gate = gate_up[2 * i];
        float up = gate_up[2 * i + 1];
        gate = fminf(gate, limit);
        up = fminf(fmaxf(up, -limit), limit);
        const float glu = gate * (1.0f / (1.0f + expf(-alpha * gate)));
        out[i] = round_f16((up + 1.0f) * glu);
    }
}

/* expert_activation_swiglu — Metal/MoE/expert.metal:380-393. */
GWO_API void gwo_act_silu(const float* gate_up, int64_t F, float* out) {
    for (int64_t i = 0; i < F; ++i) {
        const float gate = gate_up[2 * i];
        const float up = gate_up[2 * i + 1];
        const float silu = gate * (1.0f / (1.0f + expf(-gate)));
        out[i] = round_f16(silu * up);
    }
}

/* Section spans of one expert stride (GodwitManifest.expertSections). */
typedef struct {
    int64_t offset[6];
} gwo_sections;

/* ExpertRunner.apply — Runtime/ExpertRunner.swift:275-331: gate_up GEMV with
 * bias -> activation -> down GEMV with bias.  `stride` is one expert's bytes
 * in the installed layout; y[H]. `act` 0 = GPT-OSS clamped GLU, 1 = SiLU. */
GWO_API void gwo_expert_apply(const uint8_t* stride, const int64_t* section_offset,
                              int64_t H, int64_t F, int act, float limit, float alpha,
                              const float* x, float* y) {
    const uint8_t* gu_blocks = stride + section_offset[0];
    const uint8_t* gu_scales = stride + section_offset[1];
    const uint8_t* dn_blocks = stride + section_offset[2];
    const uint8_t* dn_scales = stride + section_offset[3];
    const uint16_t* gu_bias = (const uint16_t*)(stride + section_offset[4]);
    const uint16_t* dn_bias = (const uint16_t*)(stride + section_offset[5]);
    float* gub = (float*)malloc(sizeof(float) * 2 * F);
    float* dnb = (float*)malloc(sizeof(float) * H);
    float* gu = (float*)malloc(sizeof(float) * 2 * F);
    float* a = (float*)malloc(sizeof(float) * F);
    for (int64_t i = 0; i < 2 * F; ++i) gub[i] = bf16_to_f32(gu_bias[i]);
    for (int64_t i = 0; i < H; ++i) dnb[i] = bf16_to_f32(dn_bias[i]);
    gemv_rows(gu_blocks, gu_scales, gub, x, 0, 2 * F, H, gu);
    if (act == 0) gwo_act_gptoss(gu, F, limit, alpha, a);
    else gwo_act_silu(gu, F, a);
    gemv_rows(dn_blocks, dn_scales, dnb, a, 0, H, F, y);
    free(gub); free(dnb); free(gu); free(a);
}

/* The MoE half of TransformerLayer.forward — Runtime/TransformerLayer.swift:158-238
 * with ExpertRunner.applyAssignments (ExpertRunner.swift:108-182) and
 * expert_accumulate (expert.metal:107-116): route every token, then
 * out[t] += w * expert(x[t]) in (token, rank) order.
 *   strides:   pointer to expert 0 of this layer; expert e at strides + e*stride_bytes
 *   router_w:  bf16 [E, H]; router_b: bf16 [E] or NULL
 *   experts_in/weights_in: optional fixed routing [T, k] (NULL = route here)
 *   experts_out/weights_out: routing decision [T, k] (may be NULL)
 * x [T, H] floats holding the device's input values; out [T, H]. */
GWO_API void gwo_moe_layer(const uint8_t* strides, int64_t stride_bytes,
                           const int64_t* section_offset, int64_t H, int64_t F, int64_t E,
                           int k, int act, float limit, float alpha,
                           const uint16_t* router_w, const uint16_t* router_b,
                           const float* x, int64_t T,
                           const int32_t* experts_in, const float* weights_in,
                           float* out, int32_t* experts_out, float* weights_out) {
    float* logits = (float*)malloc(sizeof(float) * E);
    float* y = (float*)malloc(sizeof(float) * H);
    int32_t ex[64];
    float wt[64];
    for (int64_t t = 0; t < T; ++t) {
        const float* xt = x + t * H;
        if (experts_in) {
            for (int j = 0; j < k; ++j) { ex[j] = experts_in[t * k + j]; wt[j] = weights_in[t * k + j]; }
        } else {
            gwo_router_logits(router_w, router_b, xt, E, H, logits);
            gwo_router_select(logits, (int)E, k, ex, wt);
        }
        if (experts_out) for (int j = 0; j < k; ++j) experts_out[t * k + j] = ex[j];
        if (weights_out) for (int j = 0; j < k; ++j) weights_out[t * k + j] = wt[j];
        float* o = out + t * H;
        for (int64_t i = 0; i < H; ++i) o[i] = 0.0f;
        for (int j = 0; j < k; ++j) {
            if (ex[j] < 0) continue;
            gwo_expert_apply(strides + (int64_t)ex[j] * stride_bytes, section_offset, H, F,
                             act, limit, alpha, xt, y);
            for (int64_t i = 0; i < H; ++i) o[i] += y[i] * wt[j];
        }
    }
    free(logits);
    free(y);
}

/* Multi-threaded MoE layer over tokens (the all-cores CPU baseline of the
 * layer configs); each token is one thread's work, so results equal
 * gwo_moe_layer's. */
typedef struct {
    const uint8_t* strides; int64_t stride_bytes; const int64_t* so; int64_t H, F, E;
    int k, act; float limit, alpha; const uint16_t* rw; const uint16_t* rb;
    const float* x; int64_t t0, t1; float* out; int32_t* eo; float* wo;
} moe_job;

static void* moe_worker(void* p) {
    moe_job* j = (moe_job*)p;
    for (int64_t t = j->t0; t < j->t1; ++t)
        gwo_moe_layer(j->strides, j->stride_bytes, j->so, j->H, j->F, j->E, j->k, j->act,
                      j->limit, j->alpha, j->rw, j->rb, j->x + t * j->H, 1, NULL, NULL,
                      j->out + t * j->H, j->eo ? j->eo + t * j->k : NULL,
                      j->wo ? j->wo + t * j->k : NULL);
    return NULL;
}

GWO_API void gwo_moe_layer_mt(const uint8_t* strides, int64_t stride_bytes,
                              const int64_t* section_offset, int64_t H, int64_t F, int64_t E,
                              int k, int act, float limit, float alpha,
                              const uint16_t* router_w, const uint16_t* router_b,
                              const float* x, int64_t T, float* out, int32_t* experts_out,
                              float* weights_out, int threads) {
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    if (threads > T) threads = (int)T;
    pthread_t tid[256];
    moe_job jobs[256];
    const int64_t per = (T + threads - 1) / threads;
    int started = 0;
    for (int t = 0; t < threads; ++t) {
        const int64_t t0 = t * per, t1 = (t + 1) * per < T ? (t + 1) * per : T;
        if (t0 >= t1) break;
        jobs[t] = (moe_job){strides, stride_bytes, section_offset, H, F, E, k, act, limit, alpha,
                            router_w, router_b, x, t0, t1, out, experts_out, weights_out};
        if (pthread_create(&tid[t], NULL, moe_worker, &jobs[t]) != 0) {
            moe_worker(&jobs[t]);
            tid[t] = 0;
        }
        started = t + 1;
    }
    for (int t = 0; t < started; ++t)
        if (tid[t]) pthread_join(tid[t], NULL);
}

/* fp64 decode for the fp64 parity oracle: codebook x 2^(byte-127) (the
 * MXFP4.decode arithmetic of MXFP4.swift:48-92, carried out in double, where
 * every byte including 0xFF is a finite power of two), rows of a
 * [rows][cols] matrix, row-parallel over `threads`. */
typedef struct {
    const uint8_t* packed; const uint8_t* scales; int64_t r0, r1, cols; double* out;
} dq64_job;

static void* dq64_worker(void* p) {
    dq64_job* j = (dq64_job*)p;
    const int64_t nb = j->cols / 32;
    for (int64_t r = j->r0; r < j->r1; ++r) {
        for (int64_t b = 0; b < nb; ++b) {
            const uint8_t sb = j->scales[r * nb + b];
            const double s = ldexp(1.0, (int)sb - 127);
            const uint8_t* q = j->packed + (r * nb + b) * 16;
            double* o = j->out + r * j->cols + b * 32;
            for (int i = 0; i < 16; ++i) {
                o[2 * i] = (double)kCodebook[q[i] & 0x0F] * s;
                o[2 * i + 1] = (double)kCodebook[q[i] >> 4] * s;
            }
        }
    }
    return NULL;
}

GWO_API void gwo_dequant64_mt(const uint8_t* packed, const uint8_t* scales, int64_t rows,
                              int64_t cols, double* out, int threads) {
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    pthread_t tid[256];
    dq64_job jobs[256];
    const int64_t per = (rows + threads - 1) / threads;
    int started = 0;
    for (int t = 0; t < threads; ++t) {
        const int64_t r0 = t * per, r1 = (t + 1) * per < rows ? (t + 1) * per : rows;
        if (r0 >= r1) break;
        jobs[t] = (dq64_job){packed, scales, r0, r1, cols, out};
        if (threads == 1 || pthread_create(&tid[t], NULL, dq64_worker, &jobs[t]) != 0) {
            dq64_worker(&jobs[t]);
            tid[t] = 0;
        }
        started = t + 1;
    }
    for (int t = 0; t < started; ++t)
        if (tid[t]) pthread_join(tid[t], NULL);
}

/* ---- int8 affine trunk projections --------------------------------------
 * Int8Affine (Sources/Godwit/Install/Int8Affine.swift) quantises the trunk
 * (output head, attention projections) to one uint8 code per weight with a
 * bf16 (scale, zero) pair per group of 64 columns: codes [rows][cols], then
 * the pairs [rows][cols/64][2] (Install/Installer.swift:315-345,
 * InstallLayout.swift:151-157).  The GEMVs are router.metal:65-141. */

/* BFloat16.fromFloat — Install/Int8Affine.swift:89-96: round to nearest even,
 * NaN kept a NaN. */
GWO_API uint16_t gwo_bf16_from_f32(float v) {
    uint32_t bits;
    memcpy(&bits, &v, 4);
    if ((bits & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((bits >> 16) | 0x0040u);
    const uint32_t rounding = ((bits >> 16) & 1u) + 0x7FFFu;
    return (uint16_t)((bits + rounding) >> 16);
}

/* Int8Affine.quantize(row:) — Install/Int8Affine.swift:31-58.  Per group of
 * 64: low/high by a sequential scan, scale = max((high-low)/255,
 * FLT_MIN), zero = low, code = clamp(round((v-low)/scale), 0, 255) with
 * Swift's .rounded() (half away from zero: roundf).  Returns 0, or -1 when n
 * is not a multiple of 64 (the reference's precondition). */
GWO_API int gwo_int8_quantize_row(const float* row, int64_t n, uint8_t* codes, float* scale,
                                  float* zero) {
    if (n % 64) return -1;
    for (int64_t g = 0; g < n / 64; ++g) {
        const float* v = row + g * 64;
        float low = v[0], high = v[0];
        for (int i = 1; i < 64; ++i) {
            low = fminf(low, v[i]);
            high = fmaxf(high, v[i]);
        }
        float s = (high - low) / 255.0f;
        if (!(s >= 1.17549435e-38f)) s = 1.17549435e-38f;  /* max(_, .leastNormalMagnitude) */
        scale[g] = s;
        zero[g] = low;
        for (int i = 0; i < 64; ++i) {
            float level = roundf((v[i] - low) / s);
            level = level < 0.0f ? 0.0f : (level > 255.0f ? 255.0f : level);
            codes[g * 64 + i] = (uint8_t)level;
        }
    }
    return 0;
}

/* Int8Affine.dequantize — Install/Int8Affine.swift:61-73, with the bf16 pair
 * layout the device reads (ModelRunner.embed, Runtime/ModelRunner.swift:131-157):
 * w = code * scale + zero in fp32. */
GWO_API void gwo_int8_dequant(const uint8_t* codes, const uint16_t* meta, int64_t rows,
                              int64_t cols, float* out) {
    const int64_t ng = cols / 64;
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t g = 0; g < ng; ++g) {
            const float s = bf16_to_f32(meta[(r * ng + g) * 2]);
            const float z = bf16_to_f32(meta[(r * ng + g) * 2 + 1]);
            for (int i = 0; i < 64; ++i) {
                const int64_t c = r * cols + g * 64 + i;
                out[c] = (float)codes[c] * s + z;
            }
        }
}

/* int8_affine_gemv / int8_affine_gemv_bias_batched — Metal/MoE/router.metal:65-141:
 * per row and group, dot = sum q*x and xsum = sum x in fp32 over the 64
 * columns, acc += scale*dot + zero*xsum; y = acc (+ bias).  The Metal
 * kernel spreads the groups over 32 lanes and sums the lanes at the end;
 * this restatement walks the groups in order.  x holds the f16 values
 * [T][cols]; y [T][rows] fp32 (the batched kernel's f16 rounding is the
 * caller's).  Rows split over `threads` POSIX threads. */
typedef struct {
    const uint8_t* codes; const uint16_t* meta; const uint16_t* bias; const float* x;
    int64_t T, rows, cols, r0, r1; float* y;
} i8_job;

static void* i8_worker(void* p) {
    const i8_job* j = (const i8_job*)p;
    const int64_t ng = j->cols / 64;
    for (int64_t r = j->r0; r < j->r1; ++r) {
        const uint8_t* w = j->codes + r * j->cols;
        const uint16_t* m = j->meta + r * ng * 2;
        for (int64_t t = 0; t < j->T; ++t) {
            const float* xt = j->x + t * j->cols;
            float acc = 0.0f;
            for (int64_t g = 0; g < ng; ++g) {
                const float scale = bf16_to_f32(m[g * 2]), zero = bf16_to_f32(m[g * 2 + 1]);
                float dot = 0.0f, xsum = 0.0f;
                for (int i = 0; i < 64; ++i) {
                    const float xi = xt[g * 64 + i];
                    dot += (float)w[g * 64 + i] * xi;
                    xsum += xi;
                }
                acc += scale * dot + zero * xsum;
            }
            j->y[t * j->rows + r] = acc + (j->bias ? bf16_to_f32(j->bias[r]) : 0.0f);
        }
    }
    return NULL;
}

GWO_API void gwo_int8_gemv_mt(const uint8_t* codes, const uint16_t* meta, const uint16_t* bias,
                              const float* x, int64_t T, int64_t rows, int64_t cols, float* y,
                              int threads) {
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    pthread_t tid[256];
    i8_job jobs[256];
    const int64_t per = (rows + threads - 1) / threads;
    int started = 0;
    for (int t = 0; t < threads; ++t) {
        const int64_t r0 = t * per, r1 = (t + 1) * per < rows ? (t + 1) * per : rows;
        if (r0 >= r1) break;
        jobs[t] = (i8_job){codes, meta, bias, x, T, rows, cols, r0, r1, y};
        if (threads == 1 || pthread_create(&tid[t], NULL, i8_worker, &jobs[t]) != 0) {
            i8_worker(&jobs[t]);
            tid[t] = 0;
        }
        started = t + 1;
    }
    for (int t = 0; t < started; ++t)
        if (tid[t]) pthread_join(tid[t], NULL);
}
