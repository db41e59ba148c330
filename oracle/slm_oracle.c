/*
 * slm_oracle.c -- CPU restatement of python-slm's optimizer step.
 *
 * TEST INFRASTRUCTURE ONLY (the checker).  See slm_oracle.h for what is pinned
 * by which reference test.  Compiled with -ffp-contract=off -fno-fast-math so
 * every f32 expression below rounds once per operation, in source order, with
 * no fused multiply-add -- the same arithmetic as the reference's Rust, which
 * never contracts.
 */
#include "slm_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

static inline uint32_t f32_bits(float v) {
    uint32_t b;
    memcpy(&b, &v, 4);
    return b;
}

static inline float bits_f32(uint32_t b) {
    float v;
    memcpy(&v, &b, 4);
    return v;
}

static inline int is_finite_f32(float v) { return (f32_bits(v) & 0x7f800000u) != 0x7f800000u; }

/* src/model/oracle.rs:300-304 f32_to_bf16_bits: round to nearest even by
 * adding 0x7fff plus the lowest kept bit, then dropping the low half. */
uint16_t slmo_f32_to_bf16_bits(float value) {
    uint32_t bits = f32_bits(value);
    uint32_t rounding_bias = 0x7fffu + ((bits >> 16) & 1u);
    return (uint16_t)((bits + rounding_bias) >> 16);
}

/* src/model/oracle.rs:306-308 bf16_bits_to_f32. */
float slmo_bf16_bits_to_f32(uint16_t bits) { return bits_f32((uint32_t)bits << 16); }

/* Rust's f32::powi(base, n) with a run-time exponent lowers to LLVM's
 * llvm.powi.f32.i32, which on x86-64 becomes a call to the compiler-builtins
 * routine __powisf2 (Rust compiler-builtins crate, restating LLVM
 * compiler-rt lib/builtins/powisf2.c): square-and-multiply from the lowest
 * exponent bit, one f32 rounding per multiply, reciprocal for n < 0.  The
 * reference calls it at src/model/oracle.rs:539-540. */
float slmo_powi(float base, int32_t exponent) {
    int recip = exponent < 0;
    uint32_t remaining = recip ? (uint32_t)(-(int64_t)exponent) : (uint32_t)exponent;
    float product = 1.0f;
    for (;;) {
        if (remaining & 1u) product = product * base;
        remaining >>= 1;
        if (remaining == 0) break;
        base = base * base;
    }
    return recip ? 1.0f / product : product;
}

/* src/model/oracle.rs:486-507 gradient_clip_scale: sequential f32 sum of
 * squares, fail closed on any non-finite element or sum. */
int slmo_gradient_clip_scale(const float* gradients, uint64_t n, float* out_scale) {
    float sum = 0.0f;
    for (uint64_t i = 0; i < n; ++i) {
        float g = gradients[i];
        if (!is_finite_f32(g)) return SLMO_MODEL_GRADIENT_NONFINITE;
        sum = sum + g * g;
    }
    if (!is_finite_f32(sum)) return SLMO_MODEL_GRADIENT_NORM_NONFINITE;
    if (sum == 0.0f) {
        *out_scale = 1.0f;
        return SLMO_OK;
    }
    float scale = 1.0f / sqrtf(sum);
    *out_scale = scale < 1.0f ? scale : 1.0f;
    return SLMO_OK;
}

/* The sum inside gradient_clip_scale (src/model/oracle.rs:487-496) on its
 * own: fl(sum + fl(g * g)) in element order.  Returns
 * SLMO_MODEL_GRADIENT_NONFINITE at a non-finite element (as the reference
 * does); the sum itself may overflow to inf. */
int slmo_reference_sum_squares(const float* gradients, uint64_t n, float* out_sum) {
    float sum = 0.0f;
    for (uint64_t i = 0; i < n; ++i) {
        float g = gradients[i];
        if (!is_finite_f32(g)) return SLMO_MODEL_GRADIENT_NONFINITE;
        sum = sum + g * g;
    }
    *out_sum = sum;
    return SLMO_OK;
}

/* Constants of OPT-001, src/model/oracle.rs:469-484 optimizer_rules. */
#define RULE_BETA1 0.9f
#define RULE_BETA2 0.95f
#define RULE_EPSILON 1.0e-8f

/* The AdamW arithmetic of src/model/oracle.rs:536-543 with the bias
 * corrections (1 - beta^t) supplied by the caller.  Operation order:
 *   m' = (b1*m) + ((1-b1)*g)
 *   v' = (b2*v) + (((1-b2)*g)*g)
 *   m^ = m' / (1-b1^t)            (true division)
 *   v^ = v' / (1-b2^t)            (true division)
 *   t' = theta - lr*((m^ / (sqrt(v^) + eps)) + wd*theta)
 * Returns nonzero when any output is non-finite. */
static inline int adamw_core(float theta, float g, float m, float v, float lr, float wd,
                             float b1, float b2, float omb1, float omb2, float bc1, float bc2,
                             float eps, float* o_theta, float* o_m, float* o_v) {
    float m1 = b1 * m + omb1 * g;
    float v1 = b2 * v + omb2 * g * g;
    float mh = m1 / bc1;
    float vh = v1 / bc2;
    float denom = sqrtf(vh) + eps;
    float upd = mh / denom + wd * theta;
    float t1 = theta - lr * upd;
    *o_theta = t1;
    *o_m = m1;
    *o_v = v1;
    return !(is_finite_f32(m1) && is_finite_f32(v1) && is_finite_f32(t1));
}

/* src/model/oracle.rs:509-559 adamw_scalar_step, including its input and
 * result checks and the per-call powi. */
int slmo_adamw_scalar_step(float theta, float gradient, float moment, float variance,
                           float learning_rate, uint32_t one_based_update, float weight_decay,
                           float* out_master, float* out_moment, float* out_variance,
                           uint16_t* out_bf16) {
    if (one_based_update == 0 || !is_finite_f32(theta) || !is_finite_f32(gradient) ||
        !is_finite_f32(moment) || !is_finite_f32(variance) || !is_finite_f32(learning_rate) ||
        !is_finite_f32(weight_decay))
        return SLMO_MODEL_OPTIMIZER_INPUT_INVALID;
    const float b1 = RULE_BETA1, b2 = RULE_BETA2;
    const float omb1 = 1.0f - b1, omb2 = 1.0f - b2;
    const int32_t t = (int32_t)one_based_update;
    const float bc1 = 1.0f - slmo_powi(b1, t);
    const float bc2 = 1.0f - slmo_powi(b2, t);
    float th, m1, v1;
    if (adamw_core(theta, gradient, moment, variance, learning_rate, weight_decay, b1, b2, omb1,
                   omb2, bc1, bc2, RULE_EPSILON, &th, &m1, &v1))
        return SLMO_MODEL_OPTIMIZER_RESULT_NONFINITE;
    *out_master = th;
    *out_moment = m1;
    *out_variance = v1;
    *out_bf16 = slmo_f32_to_bf16_bits(th);
    return SLMO_OK;
}

/* src/train/trainer.rs:102-119 canonical_learning_rate, generalised over its
 * four constants: linear warmup in f32, then a cosine in f64 with the
 * (peak - minimum) difference taken in f32 first, cast back to f32. */
int slmo_schedule_learning_rate(uint64_t t, float peak, float minimum, uint64_t warmup,
                                uint64_t total, float* out) {
    if (t < 1 || t > total || warmup >= total) return SLMO_P12_SCHEDULE_INDEX_INVALID;
    if (t <= warmup) {
        *out = peak * (float)t / (float)warmup;
        return SLMO_OK;
    }
    double progress = (double)(t - warmup) / (double)(total - warmup);
    double lr = (double)minimum + 0.5 * (double)(peak - minimum) *
                                      (1.0 + cos(3.14159265358979323846 * progress));
    *out = (float)lr;
    return SLMO_OK;
}

/* src/train/trainer.rs:21-22 and :16-18: peak 0.0025, minimum 0.00025,
 * 1,000 warmup updates of 30,518. */
int slmo_canonical_learning_rate(uint64_t t, float* out) {
    return slmo_schedule_learning_rate(t, 0.0025f, 0.00025f, 1000u, 30518u, out);
}

/* ---- SHA-256, FIPS 180-4 --------------------------------------------------- */
static const uint32_t K256[64] = {
    0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u, 0x923f82a4u,
    0xab1c5ed5u, 0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u, 0x72be5d74u, 0x80deb1feu,
    0x9bdc06a7u, 0xc19bf174u, 0xe49b69c1u, 0xefbe4786u, 0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu,
    0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau, 0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u,
    0xc6e00bf3u, 0xd5a79147u, 0x06ca6351u, 0x14292967u, 0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu,
    0x53380d13u, 0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u, 0xa2bfe8a1u, 0xa81a664bu,
    0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u, 0x19a4c116u,
    0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au, 0x5b9cca4fu, 0x682e6ff3u,
    0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u, 0x90befffau, 0xa4506cebu, 0xbef9a3f7u,
    0xc67178f2u};

static inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

static void sha256_block(uint32_t h[8], const uint8_t* p) {
    uint32_t w[64];
    for (int i = 0; i < 16; ++i)
        w[i] = ((uint32_t)p[4 * i] << 24) | ((uint32_t)p[4 * i + 1] << 16) |
               ((uint32_t)p[4 * i + 2] << 8) | (uint32_t)p[4 * i + 3];
    for (int i = 16; i < 64; ++i) {
        uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
        uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
        w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], k = h[7];
    for (int i = 0; i < 64; ++i) {
        uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
        uint32_t ch = (e & f) ^ (~e & g);
        uint32_t t1 = k + S1 + ch + K256[i] + w[i];
        uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
        uint32_t mj = (a & b) ^ (a & c) ^ (b & c);
        uint32_t t2 = S0 + mj;
        k = g;
        g = f;
        f = e;
        e = d + t1;
        d = c;
        c = b;
        b = a;
        a = t1 + t2;
    }
    h[0] += a;
    h[1] += b;
    h[2] += c;
    h[3] += d;
    h[4] += e;
    h[5] += f;
    h[6] += g;
    h[7] += k;
}

void slmo_sha256_init(slmo_sha256_ctx* ctx) {
    static const uint32_t H0[8] = {0x6a09e667u, 0xbb67ae85u, 0x3c6ef372u, 0xa54ff53au,
                                   0x510e527fu, 0x9b05688cu, 0x1f83d9abu, 0x5be0cd19u};
    memcpy(ctx->h, H0, sizeof(H0));
    ctx->length = 0;
    ctx->used = 0;
}

void slmo_sha256_update(slmo_sha256_ctx* ctx, const void* data, uint64_t n) {
    const uint8_t* p = (const uint8_t*)data;
    ctx->length += n;
    if (ctx->used) {
        while (n && ctx->used < 64) {
            ctx->block[ctx->used++] = *p++;
            --n;
        }
        if (ctx->used == 64) {
            sha256_block(ctx->h, ctx->block);
            ctx->used = 0;
        }
    }
    while (n >= 64) {
        sha256_block(ctx->h, p);
        p += 64;
        n -= 64;
    }
    while (n) {
        ctx->block[ctx->used++] = *p++;
        --n;
    }
}

void slmo_sha256_final(slmo_sha256_ctx* ctx, uint8_t out[32]) {
    uint64_t bit_length = ctx->length * 8u;
    uint8_t pad = 0x80;
    slmo_sha256_update(ctx, &pad, 1);
    uint8_t zero = 0;
    while (ctx->used != 56) slmo_sha256_update(ctx, &zero, 1);
    uint8_t len_be[8];
    for (int i = 0; i < 8; ++i) len_be[i] = (uint8_t)(bit_length >> (56 - 8 * i));
    slmo_sha256_update(ctx, len_be, 8);
    for (int i = 0; i < 8; ++i) {
        out[4 * i] = (uint8_t)(ctx->h[i] >> 24);
        out[4 * i + 1] = (uint8_t)(ctx->h[i] >> 16);
        out[4 * i + 2] = (uint8_t)(ctx->h[i] >> 8);
        out[4 * i + 3] = (uint8_t)ctx->h[i];
    }
}

void slmo_sha256(const void* data, uint64_t n, uint8_t out[32]) {
    slmo_sha256_ctx ctx;
    slmo_sha256_init(&ctx);
    slmo_sha256_update(&ctx, data, n);
    slmo_sha256_final(&ctx, out);
}

/* ---- fixed-order f64 norm tree ---------------------------------------------
 * The flat gradient is cut into chunks of 65,536 elements (the last one may be
 * short; missing elements contribute nothing, which equals adding +0.0 to a
 * non-negative sum).  One chunk partial is formed exactly like a 256-thread
 * CUDA block does it:
 *   lane t (0..255) owns, for k = 0..31, the 8 consecutive elements starting
 *   at k*2048 + t*8; it squares them in f32, sums the 8 squares pairwise in
 *   f32 as ((q0+q1)+(q2+q3))+((q4+q5)+(q6+q7)) and adds that sum, in k order,
 *   to its f64 accumulator (all terms are >= 0: the partial's relative error
 *   stays below ~2.4e-7);
 *   each warp of 32 lanes folds with offsets 16,8,4,2,1 (lane l += lane l+off);
 *   the 8 warp results fold with offsets 4,2,1.
 * The total over chunk partials uses the same shape: lane t adds partials
 * t, t+256, t+512, ... in order, then the same warp and block folds.  Chunk
 * partials of zero padding are +0.0, so padding the chunk count (ZeRO-1
 * shards) leaves the total bit-identical. */
static double tree_fold(double* lane) {
    double warp[8];
    for (int w = 0; w < 8; ++w) {
        double v[32];
        for (int l = 0; l < 32; ++l) v[l] = lane[32 * w + l];
        for (int off = 16; off >= 1; off >>= 1)
            for (int l = 0; l < off; ++l) v[l] = v[l] + v[l + off];
        warp[w] = v[0];
    }
    for (int off = 4; off >= 1; off >>= 1)
        for (int i = 0; i < off; ++i) warp[i] = warp[i] + warp[i + off];
    return warp[0];
}

uint64_t slmo_chunk_count(uint64_t n) { return (n + SLMO_CHUNK_ELEMS - 1) / SLMO_CHUNK_ELEMS; }

static double chunk_partial_f32(const float* g, uint64_t n, uint64_t chunk, uint8_t* bad_out) {
    double lane[SLMO_TREE_THREADS];
    const uint64_t base = chunk * (uint64_t)SLMO_CHUNK_ELEMS;
    int bad = 0;
    for (uint32_t t = 0; t < SLMO_TREE_THREADS; ++t) {
        double acc = 0.0;
        for (uint32_t k = 0; k < SLMO_CHUNK_ELEMS / (SLMO_TREE_THREADS * SLMO_TREE_VEC); ++k) {
            uint64_t e0 = base + (uint64_t)k * SLMO_TREE_THREADS * SLMO_TREE_VEC +
                          (uint64_t)t * SLMO_TREE_VEC;
            if (e0 >= n) break;
            float q[SLMO_TREE_VEC];
            for (uint32_t j = 0; j < SLMO_TREE_VEC; ++j) {
                uint64_t e = e0 + j;
                float x = e < n ? g[e] : 0.0f;
                if (!is_finite_f32(x)) bad = 1;
                q[j] = x * x;
            }
            float p = ((q[0] + q[1]) + (q[2] + q[3])) + ((q[4] + q[5]) + (q[6] + q[7]));
            if (!is_finite_f32(p)) bad = 1;
            acc = acc + (double)p;
        }
        lane[t] = acc;
    }
    *bad_out = (uint8_t)bad;
    return tree_fold(lane);
}

void slmo_chunk_partials_f32(const float* g, uint64_t n, double* partials, uint8_t* nonfinite,
                             int threads) {
    const int64_t chunks = (int64_t)slmo_chunk_count(n);
    if (threads < 1) threads = 1;
#pragma omp parallel for num_threads(threads) schedule(static)
    for (int64_t c = 0; c < chunks; ++c)
        partials[c] = chunk_partial_f32(g, n, (uint64_t)c, &nonfinite[c]);
}

double slmo_tree_sum(const double* partials, uint64_t count) {
    double lane[SLMO_TREE_THREADS];
    for (uint32_t t = 0; t < SLMO_TREE_THREADS; ++t) {
        double s = 0.0;
        for (uint64_t c = t; c < count; c += SLMO_TREE_THREADS) s = s + partials[c];
        lane[t] = s;
    }
    return tree_fold(lane);
}

/* The reference's clip formula (src/model/oracle.rs:497-506) applied to the
 * f64 tree sum rounded once to f32:  sum == 0 -> 1, otherwise
 * min(max_norm / sqrt(sum), 1); a sum that is not finite in f32 is the
 * reference's MODEL_GRADIENT_NORM_NONFINITE. */
float slmo_clip_from_sum(double sum_squares, float max_norm, int* norm_nonfinite) {
    float sum = (float)sum_squares;
    *norm_nonfinite = !is_finite_f32(sum);
    if (*norm_nonfinite) return 0.0f;
    if (sum == 0.0f) return 1.0f;
    float scale = max_norm / sqrtf(sum);
    return scale < 1.0f ? scale : 1.0f;
}

/* ---- gradient decode ---------------------------------------------------------
 * Unscale is a true f32 division, the analogue of the reference's normalise
 * step `value / divisor` (src/train/trainer.rs:884, :892-896). */
void slmo_unscale_f32(const float* x, uint64_t n, float scale, float* out, int threads) {
    if (threads < 1) threads = 1;
#pragma omp parallel for num_threads(threads) schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) out[i] = x[i] / scale;
}

void slmo_unscale_bf16(const uint16_t* x, uint64_t n, float scale, float* out, int threads) {
    if (threads < 1) threads = 1;
#pragma omp parallel for num_threads(threads) schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) out[i] = slmo_bf16_bits_to_f32(x[i]) / scale;
}

/* ZeRO-1 gradient reduction: f32 sum of every rank's bf16 gradient in rank
 * order 0..N-1 (left to right), the analogue of the reference's micro-batch
 * accumulation `total += value` (src/train/trainer.rs:865-877). */
void slmo_rank_sum_bf16(const uint16_t* const* grads, uint32_t ranks, uint64_t n, float* out,
                        int threads) {
    if (threads < 1) threads = 1;
#pragma omp parallel for num_threads(threads) schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) {
        float s = slmo_bf16_bits_to_f32(grads[0][i]);
        for (uint32_t r = 1; r < ranks; ++r) s = s + slmo_bf16_bits_to_f32(grads[r][i]);
        out[i] = s;
    }
}

/* AdamW over local elements [0, n) whose global flat indices start at
 * elem_base (the decay weight comes from the global tensor table): unscale
 * g_raw by `scale` (true division), multiply by `clip` when cfg->apply_clip,
 * then src/model/oracle.rs:536-543 and bf16 storage.  Returns nonzero when any
 * output is non-finite.  This is the update half of the fused step; a ZeRO-1
 * rank runs it over its shard with the group's clip. */
int slmo_adamw_apply_range(const slmo_step_config* cfg, const float* g_raw, uint64_t n,
                           uint64_t elem_base, const uint64_t* tensor_offsets,
                           const uint8_t* tensor_decay, uint32_t n_tensors, float scale,
                           float clip, float* master, float* moment, float* variance,
                           uint16_t* bf16, int threads) {
    const float b1 = cfg->beta1, b2 = cfg->beta2, eps = cfg->epsilon;
    const float omb1 = 1.0f - b1, omb2 = 1.0f - b2;
    const float bc1 = 1.0f - slmo_powi(b1, (int32_t)cfg->one_based_update);
    const float bc2 = 1.0f - slmo_powi(b2, (int32_t)cfg->one_based_update);
    const float lr = cfg->learning_rate;
    const float use_clip = cfg->apply_clip ? clip : 1.0f;
    if (threads < 1) threads = 1;
    int any_bad = 0;
    const uint64_t end = elem_base + n;
    for (uint32_t k = 0; k < n_tensors; ++k) {
        uint64_t glo = tensor_offsets[k], ghi = tensor_offsets[k + 1];
        if (ghi <= elem_base || glo >= end) continue;
        if (glo < elem_base) glo = elem_base;
        if (ghi > end) ghi = end;
        const float wd = tensor_decay[k] ? cfg->decay_weight : cfg->no_decay_weight;
        const int64_t lo = (int64_t)(glo - elem_base), hi = (int64_t)(ghi - elem_base);
        int bad = 0;
#pragma omp parallel for num_threads(threads) schedule(static) reduction(| : bad) if (hi - lo > 65536)
        for (int64_t i = lo; i < hi; ++i) {
            float gv = g_raw[i] / scale;
            float gc = cfg->apply_clip ? gv * use_clip : gv;
            float th, m1, v1;
            bad |= adamw_core(master[i], gc, moment[i], variance[i], lr, wd, b1, b2, omb1, omb2,
                              bc1, bc2, eps, &th, &m1, &v1);
            master[i] = th;
            moment[i] = m1;
            variance[i] = v1;
            bf16[i] = slmo_f32_to_bf16_bits(th);
        }
        any_bad |= bad;
    }
    return any_bad;
}

/* ---- the fused step ------------------------------------------------------------
 * unscale -> non-finite check -> fixed-tree norm -> clip -> AdamW per tensor
 * (decay weight by group, src/train/trainer.rs:274-293 with :276) -> bf16
 * storage, plus the dynamic loss-scale policy: skip and halve on a non-finite
 * gradient, double after growth_interval consecutive applied steps. */
int slmo_step(const slmo_step_config* cfg, const void* grads, int dtype, uint64_t n,
              const uint64_t* tensor_offsets, const uint8_t* tensor_decay, uint32_t n_tensors,
              float* master, float* moment, float* variance, uint16_t* bf16,
              slmo_scaler* scaler, slmo_step_result* out, int threads) {
    memset(out, 0, sizeof(*out));
    if (!cfg || !grads || n == 0 || n_tensors == 0 || tensor_offsets[0] != 0 ||
        tensor_offsets[n_tensors] != n || cfg->one_based_update == 0 ||
        !is_finite_f32(cfg->learning_rate) || (dtype != SLMO_DTYPE_F32 && dtype != SLMO_DTYPE_BF16))
        return out->status = SLMO_INVALID_ARGUMENT;
    if (cfg->loss_scale_mode == SLMO_SCALE_DYNAMIC && !scaler)
        return out->status = SLMO_INVALID_ARGUMENT;
    if (threads < 1) threads = 1;
    const float scale =
        cfg->loss_scale_mode == SLMO_SCALE_DYNAMIC ? scaler->scale : cfg->static_loss_scale;
    out->loss_scale_used = scale;
    out->next_loss_scale = scale;

    float* g = (float*)malloc(n * sizeof(float));
    const uint64_t chunks = slmo_chunk_count(n);
    double* partials = (double*)malloc(chunks * sizeof(double));
    uint8_t* flags = (uint8_t*)malloc(chunks);
    if (!g || !partials || !flags) {
        free(g);
        free(partials);
        free(flags);
        return out->status = SLMO_INVALID_ARGUMENT;
    }
    if (dtype == SLMO_DTYPE_F32)
        slmo_unscale_f32((const float*)grads, n, scale, g, threads);
    else
        slmo_unscale_bf16((const uint16_t*)grads, n, scale, g, threads);
    slmo_chunk_partials_f32(g, n, partials, flags, threads);
    int nonfinite = 0;
    for (uint64_t c = 0; c < chunks; ++c) nonfinite |= flags[c];
    double sum = slmo_tree_sum(partials, chunks);
    int norm_bad = 0;
    float clip = slmo_clip_from_sum(sum, cfg->max_grad_norm, &norm_bad);
    out->sum_squares = sum;
    out->grad_norm = sqrt(sum);
    out->clip_scale = clip;
    out->nonfinite = (uint32_t)nonfinite;

    if (nonfinite || norm_bad) {
        out->skipped = 1;
        if (cfg->nonfinite_policy == SLMO_NONFINITE_ERROR)
            out->status =
                nonfinite ? SLMO_MODEL_GRADIENT_NONFINITE : SLMO_MODEL_GRADIENT_NORM_NONFINITE;
        if (cfg->loss_scale_mode == SLMO_SCALE_DYNAMIC) {
            scaler->scale = scale * 0.5f;
            scaler->good_steps = 0;
        }
    } else if (cfg->min_clip_accept > 0.0f && clip < cfg->min_clip_accept) {
        out->skipped = 1;
        out->rejected = 1;
        out->status = SLMO_P12_OPTIMIZER_GRADIENT_INVALID;
    } else {
        /* g is already unscaled: apply with scale 1 (x / 1 == x exactly). */
        const int any_bad = slmo_adamw_apply_range(cfg, g, n, 0, tensor_offsets, tensor_decay,
                                                   n_tensors, 1.0f, clip, master, moment,
                                                   variance, bf16, threads);
        out->result_nonfinite = (uint32_t)any_bad;
        if (any_bad) out->status = SLMO_MODEL_OPTIMIZER_RESULT_NONFINITE;
        if (cfg->loss_scale_mode == SLMO_SCALE_DYNAMIC) {
            scaler->good_steps += 1;
            if (scaler->good_steps >= cfg->growth_interval) {
                scaler->scale = scale * 2.0f;
                scaler->good_steps = 0;
            }
        }
    }
    if (cfg->loss_scale_mode == SLMO_SCALE_DYNAMIC) {
        out->next_loss_scale = scaler->scale;
        out->good_steps = scaler->good_steps;
    }
    free(g);
    free(partials);
    free(flags);
    return out->status;
}

/* src/train/trainer.rs:222-295 CanonicalAdamw::apply_normalized_clipped_gradients:
 * length check, clip re-verification (tolerance 0.05, trainer.rs:161), u32
 * update index, frozen-schedule lr bits, then the scalar loop in PARAM-001
 * order with decay 0.1 / 0.0 by group (:276).  A mid-loop error leaves the
 * earlier elements updated, as the reference does. */
int slmo_apply_normalized_clipped_gradients(const float* gradients, uint64_t n,
                                            float learning_rate, uint64_t one_based_update,
                                            const uint64_t* tensor_offsets,
                                            const uint8_t* tensor_decay, uint32_t n_tensors,
                                            float* master, float* moment, float* variance,
                                            uint16_t* bf16, float* out_observed_clip) {
    if (n_tensors == 0 || tensor_offsets[n_tensors] != n) return SLMO_P12_OPTIMIZER_GRADIENT_INVALID;
    float observed = 0.0f;
    int st = slmo_gradient_clip_scale(gradients, n, &observed);
    if (st) return st;
    if (out_observed_clip) *out_observed_clip = observed;
    const float tolerance = 0.05f;
    if (observed < 1.0f - tolerance) return SLMO_P12_OPTIMIZER_GRADIENT_INVALID;
    if (one_based_update > 0xffffffffull) return SLMO_P12_UPDATE_INDEX_INVALID;
    float expected = 0.0f;
    st = slmo_canonical_learning_rate(one_based_update, &expected);
    if (st) return st;
    if (f32_bits(learning_rate) != f32_bits(expected)) return SLMO_P12_SCHEDULER_STATE_MISMATCH;
    for (uint32_t k = 0; k < n_tensors; ++k) {
        const float decay = tensor_decay[k] ? 0.1f : 0.0f;
        for (uint64_t i = tensor_offsets[k]; i < tensor_offsets[k + 1]; ++i) {
            float th, m1, v1;
            uint16_t b;
            st = slmo_adamw_scalar_step(master[i], gradients[i], moment[i], variance[i],
                                        learning_rate, (uint32_t)one_based_update, decay, &th, &m1,
                                        &v1, &b);
            if (st) return st;
            master[i] = th;
            moment[i] = m1;
            variance[i] = v1;
            bf16[i] = b;
        }
    }
    return SLMO_OK;
}

/* src/train/trainer.rs:297-320 CanonicalAdamw::state_sha256, with the
 * per-parameter validation of :163-189 (non-empty, finite, bf16 == RNE(master)). */
int slmo_state_sha256(const char* const* names, const uint64_t* tensor_offsets,
                      const uint8_t* tensor_decay, uint32_t n_tensors, const float* master,
                      const uint16_t* bf16, const float* moment, const float* variance,
                      char out_hex[65]) {
    static const char tag[] = "python-slm/adamw-state/v1";
    slmo_sha256_ctx ctx;
    slmo_sha256_init(&ctx);
    slmo_sha256_update(&ctx, tag, sizeof(tag)); /* includes the trailing NUL */
    for (uint32_t k = 0; k < n_tensors; ++k) {
        const uint64_t lo = tensor_offsets[k], hi = tensor_offsets[k + 1];
        const uint64_t count = hi - lo;
        const uint64_t name_len = (uint64_t)strlen(names[k]);
        if (name_len == 0 || count == 0) return SLMO_P12_OPTIMIZER_STATE_INVALID;
        for (uint64_t i = lo; i < hi; ++i) {
            if (!is_finite_f32(master[i]) || !is_finite_f32(moment[i]) ||
                !is_finite_f32(variance[i]) || slmo_f32_to_bf16_bits(master[i]) != bf16[i])
                return SLMO_P12_OPTIMIZER_STATE_INVALID;
        }
        uint8_t le[8];
        for (int b = 0; b < 8; ++b) le[b] = (uint8_t)(name_len >> (8 * b));
        slmo_sha256_update(&ctx, le, 8);
        slmo_sha256_update(&ctx, names[k], name_len);
        uint8_t decay = tensor_decay[k] ? 1 : 0;
        slmo_sha256_update(&ctx, &decay, 1);
        for (int b = 0; b < 8; ++b) le[b] = (uint8_t)(count >> (8 * b));
        slmo_sha256_update(&ctx, le, 8);
        /* x86-64 is little-endian: the in-memory bytes are the LE encoding. */
        slmo_sha256_update(&ctx, master + lo, count * 4);
        slmo_sha256_update(&ctx, bf16 + lo, count * 2);
        slmo_sha256_update(&ctx, moment + lo, count * 4);
        slmo_sha256_update(&ctx, variance + lo, count * 4);
    }
    uint8_t digest[32];
    slmo_sha256_final(&ctx, digest);
    static const char hexd[] = "0123456789abcdef";
    for (int i = 0; i < 32; ++i) {
        out_hex[2 * i] = hexd[digest[i] >> 4];
        out_hex[2 * i + 1] = hexd[digest[i] & 15];
    }
    out_hex[64] = 0;
    return SLMO_OK;
}
