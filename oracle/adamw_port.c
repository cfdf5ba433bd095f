/* TEST INFRASTRUCTURE ONLY (oracle). Never linked into the product library;
 * only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load it,
 * and only as the checker.
 *
 * Plain-C restatement ("port") of the reference's optimizer-step path, written
 * from reading the reference's src/optim/adamw.cpp, plus the pieces the reference
 * lacks (bf16 storage, loss-scale unscale, inf/NaN detect, dynamic scaler,
 * per-tensor weight decay, fp32 master weights) specified here.
 *
 * Pinning: the fp32 AdamW / clip / cosine functions are checked bit-for-bit
 * against the reference's own compiled adamw.cpp (oracle/_ref, see
 * oracle/Makefile) and against the known answers of the reference's
 * tests/test_optimizers.cpp:12-49 and :97-119 (tests/test_oracle.py). The
 * mixed-precision composite reduces to the reference code exactly (bf16->fp32
 * and power-of-two unscale are exact), which tests/test_oracle.py also checks
 * by routing the unscaled grads through the reference itself. The loss-scaler
 * state machine has no counterpart in the reference: parity there is
 * "unpinned" beyond this restatement.
 *
 * Floating-point discipline: compiled with -ffp-contract=off and no fast-math,
 * every expression keeps the reference's association so results are the same
 * bits the reference produces on x86-64 (SSE, no FMA).
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

/* ---- bf16 storage ------------------------------------------------------- */

/* bf16 -> fp32 is exact: the bf16 bits are the top half of the fp32 bits. */
float oracle_bf16_to_f32(uint16_t h) {
    uint32_t u = ((uint32_t)h) << 16;
    float f;
    memcpy(&f, &u, sizeof f);
    return f;
}

/* fp32 -> bf16, round to nearest even; any NaN becomes the canonical 0x7FFF
 * (the hardware cvt.rn.bf16.f32 result). Overflow past the bf16 max rounds to
 * inf, subnormals round like normals (no flush). */
uint16_t oracle_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, sizeof u);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)0x7FFFu;
    uint32_t lsb = (u >> 16) & 1u;
    return (uint16_t)((u + 0x7FFFu + lsb) >> 16);
}

void oracle_f32_to_bf16_array(const float* in, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = oracle_f32_to_bf16(in[i]);
}

void oracle_bf16_to_f32_array(const uint16_t* in, float* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = oracle_bf16_to_f32(in[i]);
}

/* ---- AdamW (reference src/optim/adamw.cpp) ------------------------------ */

/* adamw.cpp:68-71: bias corrections for step t (t already incremented). */
void oracle_adamw_coeffs(float lr, float beta1, float beta2, uint64_t t,
                         float* step_size, float* sqrt_bc2) {
    float bias_correction1 = 1.0f - powf(beta1, (float)t);
    float bias_correction2 = 1.0f - powf(beta2, (float)t);
    *sqrt_bc2 = sqrtf(bias_correction2);
    *step_size = lr / bias_correction1;
}

/* adamw.cpp:90-108: the per-element update of one tensor, in place. */
void oracle_adamw_update_f32(float* theta, const float* g, float* m, float* v, size_t n,
                             float lr, float beta1, float beta2, float eps, float wd,
                             float step_size, float sqrt_bc2) {
    for (size_t i = 0; i < n; ++i) {
        float g_val = g[i];
        if (wd != 0.0f) {
            theta[i] -= lr * wd * theta[i];
        }
        m[i] = beta1 * m[i] + (1.0f - beta1) * g_val;
        v[i] = beta2 * v[i] + (1.0f - beta2) * g_val * g_val;
        float denom = (sqrtf(v[i]) / sqrt_bc2) + eps;
        theta[i] -= step_size * (m[i] / denom);
    }
}

/* adamw.cpp:29-40: running double sum of squares, serial, in tensor order.
 * Returns acc + sum_i g[i]^2. */
double oracle_sumsq_f32(const float* g, size_t n, double acc) {
    for (size_t i = 0; i < n; ++i) acc += (double)g[i] * (double)g[i];
    return acc;
}

/* adamw.cpp:42 */
float oracle_norm_from_sumsq(double total_norm_sq) { return (float)sqrt(total_norm_sq); }

/* adamw.cpp:43-44: returns the clip coefficient, or 1 (no clip). */
float oracle_clip_coef(float total_norm, float max_norm, int* clipped) {
    if (total_norm > max_norm && total_norm > 1e-6f) {
        *clipped = 1;
        return max_norm / total_norm;
    }
    *clipped = 0;
    return 1.0f;
}

/* adamw.cpp:49-51 */
void oracle_scale_f32(float* g, size_t n, float coef) {
    for (size_t i = 0; i < n; ++i) g[i] *= coef;
}

/* CosineAnnealingLR::step, adamw.cpp:123-142. current_step is the value after
 * the increment; base_lr is the optimizer lr at scheduler construction. */
float oracle_cosine_lr(float base_lr, float eta_min, uint64_t total_steps,
                       uint64_t warmup_steps, uint64_t current_step) {
    if (current_step <= warmup_steps && warmup_steps > 0) {
        return base_lr * (float)current_step / (float)warmup_steps;
    }
    uint64_t adjusted_step = current_step - warmup_steps;
    uint64_t adjusted_total = total_steps - warmup_steps;
    if (adjusted_step > adjusted_total) return eta_min;
    const float pi = 3.14159265358979323846f;
    float progress = (float)adjusted_step / (float)adjusted_total;
    return eta_min + 0.5f * (base_lr - eta_min) * (1.0f + cosf(progress * pi));
}

/* ---- pieces the reference lacks ----------------------------------------- */

/* Loss-scale unscale of bf16 grads into fp32: g = float(g_bf16) * inv_scale.
 * Returns 1 when any unscaled value is inf or NaN. */
int oracle_unscale_bf16(const uint16_t* g, size_t n, float inv_scale, float* out) {
    int found = 0;
    for (size_t i = 0; i < n; ++i) {
        float x = oracle_bf16_to_f32(g[i]) * inv_scale;
        out[i] = x;
        if (!isfinite(x)) found = 1;
    }
    return found;
}

int oracle_unscale_f32(const float* g, size_t n, float inv_scale, float* out) {
    int found = 0;
    for (size_t i = 0; i < n; ++i) {
        float x = g[i] * inv_scale;
        out[i] = x;
        if (!isfinite(x)) found = 1;
    }
    return found;
}

/* Step bookkeeping shared by the device and this oracle. */
typedef struct {
    float scale;          /* current loss scale (1 when no scaler) */
    int32_t tracker;      /* clean steps since the last scale change */
    uint64_t t;           /* AdamW step_count_ (skipped steps do not count) */
    uint64_t skipped;     /* number of skipped steps */
    float last_norm;      /* pre-clip global grad norm of the last step */
    int32_t last_found_inf;
    float last_clip_coef;
} oracle_step_state;

/* Dynamic loss scaler: on inf/NaN the step is skipped, scale *= backoff and the
 * tracker resets; otherwise tracker++ and after growth_interval clean steps
 * scale *= growth and the tracker resets. */
void oracle_scaler_update(oracle_step_state* st, int found_inf, float growth_factor,
                          float backoff_factor, int32_t growth_interval) {
    if (found_inf) {
        st->scale = st->scale * backoff_factor;
        st->tracker = 0;
    } else {
        st->tracker += 1;
        if (st->tracker == growth_interval) {
            st->scale = st->scale * growth_factor;
            st->tracker = 0;
        }
    }
}

/* Sum of squares of the unscaled gradients of a tensor list, serial in tensor
 * order (adamw.cpp:29-40 on the unscaled grads). *found_inf is set when any
 * unscaled value is non-finite. scratch must hold max(numel) floats. */
double oracle_grad_sumsq(int layout, int n_tensors, void** grads, const uint64_t* numel,
                         float inv_scale, int* found_inf, float* scratch) {
    double sumsq = 0.0;
    int found = 0;
    for (int k = 0; k < n_tensors; ++k) {
        if (!grads[k] || numel[k] == 0) continue;
        int f = layout == 1
                    ? oracle_unscale_bf16((const uint16_t*)grads[k], numel[k], inv_scale, scratch)
                    : oracle_unscale_f32((const float*)grads[k], numel[k], inv_scale, scratch);
        found |= f;
        sumsq = oracle_sumsq_f32(scratch, numel[k], sumsq);
    }
    *found_inf = found;
    return sumsq;
}

/* The update half of a step, given the global sum of squares (from this
 * process alone, or summed over data-parallel ranks): skip decision, clip,
 * AdamW with the tensor's own wd, bf16 write-back, scaler update.
 * Returns 1 when the step was skipped. */
int oracle_apply_with_sumsq(int layout, int n_tensors, void** params, void** grads,
                            float** master, float** m, float** v, const uint64_t* numel,
                            const float* wd, float lr, float beta1, float beta2, float eps,
                            float max_norm, int use_scaler, float growth_factor,
                            float backoff_factor, int32_t growth_interval, double sumsq,
                            oracle_step_state* st, float* scratch) {
    float inv_scale = use_scaler ? 1.0f / st->scale : 1.0f;
    int found_inf = !isfinite(sumsq);
    float norm = oracle_norm_from_sumsq(sumsq);
    st->last_norm = norm;
    st->last_found_inf = found_inf;
    if (use_scaler && found_inf) {
        st->skipped += 1;
        st->last_clip_coef = 1.0f;
        oracle_scaler_update(st, 1, growth_factor, backoff_factor, growth_interval);
        return 1;
    }
    int clipped = 0;
    float coef = max_norm > 0.0f ? oracle_clip_coef(norm, max_norm, &clipped) : 1.0f;
    st->last_clip_coef = coef;

    st->t += 1;
    float step_size, sqrt_bc2;
    oracle_adamw_coeffs(lr, beta1, beta2, st->t, &step_size, &sqrt_bc2);
    for (int k = 0; k < n_tensors; ++k) {
        if (!grads[k] || numel[k] == 0) continue;
        size_t n = numel[k];
        if (layout == 1) oracle_unscale_bf16((const uint16_t*)grads[k], n, inv_scale, scratch);
        else oracle_unscale_f32((const float*)grads[k], n, inv_scale, scratch);
        if (clipped) oracle_scale_f32(scratch, n, coef);
        float* theta = layout == 1 ? master[k] : (float*)params[k];
        oracle_adamw_update_f32(theta, scratch, m[k], v[k], n, lr, beta1, beta2, eps, wd[k],
                                step_size, sqrt_bc2);
        if (layout == 1) oracle_f32_to_bf16_array(theta, (uint16_t*)params[k], n);
    }
    if (use_scaler) oracle_scaler_update(st, 0, growth_factor, backoff_factor, growth_interval);
    return 0;
}

/* One complete optimizer step over a tensor list, as the fused device step
 * defines it:
 *   inv = 1/scale; g = unscale(grad) (exact for power-of-two scales);
 *   found_inf = any(!isfinite(g)); skip the whole step when the scaler is on
 *   and found_inf; norm/clip exactly as AdamW::clip_grad_norm on g (when
 *   max_norm > 0); AdamW::step on the fp32 master with the tensor's own wd;
 *   bf16 params = RNE(master) in the mixed layout; scaler update.
 * layout 0: params/grads are fp32 (params are the master, updated in place).
 * layout 1: params/grads are bf16, master holds the fp32 weights.
 * Tensors with a NULL grad are skipped (adamw.cpp:30-31,74-75).
 * scratch must hold max(numel) floats. Returns 1 when the step was skipped.
 * (found_inf is carried by the sum itself: any non-finite unscaled value
 * makes the fp64 sum of squares non-finite.) */
int oracle_step(int layout, int n_tensors, void** params, void** grads, float** master,
                float** m, float** v, const uint64_t* numel, const float* wd,
                float lr, float beta1, float beta2, float eps, float max_norm,
                int use_scaler, float growth_factor, float backoff_factor,
                int32_t growth_interval, oracle_step_state* st, float* scratch) {
    float inv_scale = use_scaler ? 1.0f / st->scale : 1.0f;
    int found_inf = 0;
    double sumsq = oracle_grad_sumsq(layout, n_tensors, grads, numel, inv_scale, &found_inf,
                                     scratch);
    return oracle_apply_with_sumsq(layout, n_tensors, params, grads, master, m, v, numel, wd, lr,
                                   beta1, beta2, eps, max_norm, use_scaler, growth_factor,
                                   backoff_factor, growth_interval, sumsq, st, scratch);
}

/* ---- SGD (reference src/optim/sgd.cpp:52-96) ---------------------------- */

/* One tensor's SGD::step body (sgd.cpp:70-88); has_buf: the momentum buffer
 * holds a previous step (has_momentum_buffer_, sgd.cpp:90). */
void oracle_sgd_update_f32(float* theta, const float* grad, float* buf, size_t n, float lr,
                           float momentum, float dampening, float weight_decay, int nesterov,
                           int has_buf) {
    for (size_t i = 0; i < n; ++i) {
        float d_p = grad[i];
        if (weight_decay != 0.0f) {
            d_p += weight_decay * theta[i];
        }
        if (momentum != 0.0f) {
            if (!has_buf) {
                buf[i] = d_p;
            } else {
                buf[i] = momentum * buf[i] + (1.0f - dampening) * d_p;
            }
            if (nesterov) {
                d_p = d_p + momentum * buf[i];
            } else {
                d_p = buf[i];
            }
        }
        theta[i] -= lr * d_p;
    }
}

/* The SGD step as the fused device step defines it (unscale, inf skip, clip,
 * per-tensor wd, fp32 master, bf16 write-back, scaler), given the global sum
 * of squares. buf[k]: momentum buffers. Returns 1 when skipped. */
int oracle_sgd_apply_with_sumsq(int layout, int n_tensors, void** params, void** grads,
                                float** master, float** buf, const uint64_t* numel,
                                const float* wd, float lr, float momentum, float dampening,
                                int nesterov, float max_norm, int use_scaler, float growth_factor,
                                float backoff_factor, int32_t growth_interval, double sumsq,
                                oracle_step_state* st, float* scratch) {
    float inv_scale = use_scaler ? 1.0f / st->scale : 1.0f;
    int found_inf = !isfinite(sumsq);
    float norm = oracle_norm_from_sumsq(sumsq);
    st->last_norm = norm;
    st->last_found_inf = found_inf;
    if (use_scaler && found_inf) {
        st->skipped += 1;
        st->last_clip_coef = 1.0f;
        oracle_scaler_update(st, 1, growth_factor, backoff_factor, growth_interval);
        return 1;
    }
    int clipped = 0;
    float coef = max_norm > 0.0f ? oracle_clip_coef(norm, max_norm, &clipped) : 1.0f;
    st->last_clip_coef = coef;
    int has_buf = st->t > 0;
    st->t += 1;
    for (int k = 0; k < n_tensors; ++k) {
        if (!grads[k] || numel[k] == 0) continue;
        size_t n = numel[k];
        if (layout == 1) oracle_unscale_bf16((const uint16_t*)grads[k], n, inv_scale, scratch);
        else oracle_unscale_f32((const float*)grads[k], n, inv_scale, scratch);
        if (clipped) oracle_scale_f32(scratch, n, coef);
        float* theta = layout == 1 ? master[k] : (float*)params[k];
        oracle_sgd_update_f32(theta, scratch, buf[k], n, lr, momentum, dampening, wd[k], nesterov,
                              has_buf);
        if (layout == 1) oracle_f32_to_bf16_array(theta, (uint16_t*)params[k], n);
    }
    if (use_scaler) oracle_scaler_update(st, 0, growth_factor, backoff_factor, growth_interval);
    return 0;
}

/* ModelEMA::update (reference include/soar/utils/ema.hpp:18-28) over one
 * weight array: shadow = decay * shadow + (1 - decay) * weight. */
void oracle_ema_update(float* shadow, const float* weight, size_t n, float decay) {
    for (size_t j = 0; j < n; ++j) shadow[j] = decay * shadow[j] + (1.0f - decay) * weight[j];
}

/* ---- data-parallel reduce (ZeRO-1 reduce-scatter of bf16 gradients) ----- */

/* Average of R bf16 gradient buffers, summed in fp32 in rank order 0..R-1,
 * multiplied by 1/R once and rounded to bf16 once. This is the definition the
 * fused peer-memory reduce-scatter implements; NCCL's own reduction order is
 * implementation-defined, so the NCCL path is checked within bf16 rounding. */
void oracle_reduce_avg_bf16(int R, const uint16_t** inputs, size_t n, uint16_t* out) {
    float inv_r = 1.0f / (float)R;
    for (size_t i = 0; i < n; ++i) {
        float s = 0.0f;
        for (int r = 0; r < R; ++r) s += oracle_bf16_to_f32(inputs[r][i]);
        out[i] = oracle_f32_to_bf16(s * inv_r);
    }
}
