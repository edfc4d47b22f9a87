/*
 * oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C, fp32 restatement of teenyformers' attention-path kernels, used as
 * the parity checker for the sm_100a kernels in teenyformers_b200/csrc and as
 * the timed CPU baseline in bench.py.  Nothing in the product path links,
 * loads or calls this file; only tests/, __graft_entry__.smoke() and bench.py
 * (cpu_baseline leg and --impl reference) do.
 *
 * The reference is Rust DSL code compiled by an absent rustc fork, so it can
 * not be built or run here.  Each function below follows the reference
 * kernel's arithmetic line by line (citations are path:line inside the
 * teenyformers project):
 *
 *   orc_flash_attn2_fwd   src/kernels/flash_attn2.rs:77-125  (causal fwd; the
 *                         non-causal fwd lives in the absent teeny-kernels
 *                         crate, restated as the same loop without the mask)
 *   orc_flash_attn2_bwd   src/kernels/flash_attn2.rs:155-202 (causal) and
 *                         :229-278 (non-causal).  The reference accumulates
 *                         dK/dV with fp32 atomics in arbitrary order; here the
 *                         same sums are taken in a fixed order (one pass per
 *                         query row for dQ, one per key row for dK/dV).
 *   orc_rope              src/kernels/rope.rs:68-96 (fwd), :116-139 (bwd);
 *                         theta from ln(base) exactly as rope.rs:86-93, with
 *                         ln(base) pre-computed by the caller (rope.rs:194).
 *   orc_transpose_heads   src/kernels/transpose_heads.rs:59-70
 *   orc_merge_heads       src/kernels/transpose_heads.rs:86-95
 *   orc_rmsnorm           src/kernels/fused_add_rmsnorm.rs:53-110 (residual
 *                         optional: the layers' teeny-core RmsNorm)
 *   orc_swiglu            src/kernels/swiglu.rs:56-95
 *
 * Pinning: RoPE, RMSNorm and SwiGLU are pinned to the reference's own golden
 * vectors (tests/fixtures/{rope,fused_add_rmsnorm,swiglu},
 * tests/kernel_execution.rs:63-215).  Attention
 * forward/backward and transpose/merge: parity unpinned against the
 * reference itself (its kernels cannot be built or run here and its tests
 * hold no attention fixture); they are cross-checked against a float64
 * torch witness and numpy instead (tests/test_oracle_pinning.py).
 *
 * Generalisations (same per-sequence maths):
 *   - batch: the reference has no batch axis; [B,S,H,D] applies the
 *     reference per b.
 *   - GQA: the reference ignores n_kv_heads; query head h reads KV head
 *     h / (Hq / Hkv).
 *   - rotate-half RoPE pairs (k, k + D/2) with the reference's theta.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_EXPORT __attribute__((visibility("default")))

ORC_EXPORT int orc_version(void) { return 1; }

ORC_EXPORT int orc_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

ORC_EXPORT void orc_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

static inline int kv_head_of(int bh_q, int Hq, int Hkv) {
    int b = bh_q / Hq, h = bh_q % Hq;
    return b * Hkv + h / (Hq / Hkv);
}

/*
 * Forward, one query row at a time (flash_attn2.rs:77-125):
 *   qk = (q . k) * scale, future keys (k_row > q_row, top-left aligned,
 *   :103-107) -> -inf, online max/sum/acc (:109-115), O = acc / l,
 *   LSE = m + ln(l) (natural log of the scaled scores, :120-122).
 * Layout: q,o [B*Hq, Sq, D]; k,v [B*Hkv, Sk, D]; lse [B*Hq, Sq].
 * q_lo/q_hi restrict the rows computed (a bounded sample for timing);
 * bh_lo/bh_hi restrict the heads.
 */
ORC_EXPORT void orc_flash_attn2_fwd_range(const float* q, const float* k, const float* v,
                                          float* o, float* lse, int B, int Hq, int Hkv,
                                          int Sq, int Sk, int D, float scale, int causal,
                                          int bh_lo, int bh_hi, int q_lo, int q_hi) {
    (void)B;
    const int nrow = q_hi - q_lo;
    const long total = (long)(bh_hi - bh_lo) * nrow;
#pragma omp parallel
    {
        float* acc = (float*)malloc(sizeof(float) * (size_t)D);
#pragma omp for schedule(dynamic, 16)
        for (long t = 0; t < total; ++t) {
            const int bh = bh_lo + (int)(t / nrow);
            const int qr = q_lo + (int)(t % nrow);
            const int bkv = kv_head_of(bh, Hq, Hkv);
            const float* qv = q + ((size_t)bh * Sq + qr) * D;
            const float* kb = k + (size_t)bkv * Sk * D;
            const float* vb = v + (size_t)bkv * Sk * D;
            float m = -INFINITY, l = 0.0f;
            for (int d = 0; d < D; ++d) acc[d] = 0.0f;
            for (int kr = 0; kr < Sk; ++kr) {
                const float* kv = kb + (size_t)kr * D;
                const float* vv = vb + (size_t)kr * D;
                float dot = 0.0f;
                for (int d = 0; d < D; ++d) dot += qv[d] * kv[d];
                float qk = dot * scale;
                if (causal && kr > qr) qk = -INFINITY;
                const float m_new = fmaxf(m, qk);
                const float e_diff = expf(m - m_new);
                const float p = expf(qk - m_new);
                l = e_diff * l + p;
                for (int d = 0; d < D; ++d) acc[d] = e_diff * acc[d] + p * vv[d];
                m = m_new;
            }
            float* ov = o + ((size_t)bh * Sq + qr) * D;
            for (int d = 0; d < D; ++d) ov[d] = acc[d] / l;
            lse[(size_t)bh * Sq + qr] = m + logf(l);
        }
        free(acc);
    }
}

ORC_EXPORT void orc_flash_attn2_fwd(const float* q, const float* k, const float* v, float* o,
                                    float* lse, int B, int Hq, int Hkv, int Sq, int Sk, int D,
                                    float scale, int causal) {
    orc_flash_attn2_fwd_range(q, k, v, o, lse, B, Hq, Hkv, Sq, Sk, D, scale, causal, 0, B * Hq,
                              0, Sq);
}

/*
 * Backward (flash_attn2.rs:155-202 causal, :229-278 non-causal):
 *   D_q = sum(O_q * dO_q) (:171); per key: p = exp(qk*scale - L_q), future
 *   keys p = 0 (:186-189); ds = p * (dO_q . v_k - D_q) (:191-192);
 *   dQ_q += ds * k * scale (:194); dV_k += p * dO_q; dK_k += ds * q * scale
 *   (:196-197).  dK/dV of a KV head sum over every query head of its group.
 */
ORC_EXPORT void orc_flash_attn2_bwd(const float* q, const float* k, const float* v,
                                    const float* o, const float* dO, const float* lse,
                                    float* dq, float* dk, float* dv, int B, int Hq, int Hkv,
                                    int Sq, int Sk, int D, float scale, int causal) {
    const int G = Hq / Hkv;
    const long nq_rows = (long)B * Hq * Sq;
    float* delta = (float*)malloc(sizeof(float) * (size_t)(nq_rows > 0 ? nq_rows : 1));
#pragma omp parallel for schedule(static)
    for (long r = 0; r < nq_rows; ++r) {
        const float* ov = o + (size_t)r * D;
        const float* gv = dO + (size_t)r * D;
        float s = 0.0f;
        for (int d = 0; d < D; ++d) s += ov[d] * gv[d];
        delta[r] = s;
    }
    /* dQ: one pass per query row. */
#pragma omp parallel for schedule(dynamic, 16)
    for (long r = 0; r < nq_rows; ++r) {
        const int bh = (int)(r / Sq), qr = (int)(r % Sq);
        const int bkv = kv_head_of(bh, Hq, Hkv);
        const float* qv = q + (size_t)r * D;
        const float* gv = dO + (size_t)r * D;
        const float lq = lse[r], dq_r = delta[r];
        float* out = dq + (size_t)r * D;
        for (int d = 0; d < D; ++d) out[d] = 0.0f;
        for (int kr = 0; kr < Sk; ++kr) {
            if (causal && kr > qr) continue;
            const float* kv = k + ((size_t)bkv * Sk + kr) * D;
            const float* vv = v + ((size_t)bkv * Sk + kr) * D;
            float dot = 0.0f, dov = 0.0f;
            for (int d = 0; d < D; ++d) { dot += qv[d] * kv[d]; dov += gv[d] * vv[d]; }
            const float p = expf(dot * scale - lq);
            const float ds = p * (dov - dq_r);
            for (int d = 0; d < D; ++d) out[d] += ds * kv[d] * scale;
        }
    }
    /* dK, dV: one pass per key row, over every query of the KV head's group. */
    const long nk_rows = (long)B * Hkv * Sk;
#pragma omp parallel for schedule(dynamic, 16)
    for (long r = 0; r < nk_rows; ++r) {
        const int bkv = (int)(r / Sk), kr = (int)(r % Sk);
        const int b = bkv / Hkv, hk = bkv % Hkv;
        const float* kv = k + (size_t)r * D;
        const float* vv = v + (size_t)r * D;
        float* gk = dk + (size_t)r * D;
        float* gvv = dv + (size_t)r * D;
        for (int d = 0; d < D; ++d) { gk[d] = 0.0f; gvv[d] = 0.0f; }
        for (int g = 0; g < G; ++g) {
            const int bh = b * Hq + hk * G + g;
            for (int qr = 0; qr < Sq; ++qr) {
                if (causal && kr > qr) continue;
                const size_t qi = (size_t)bh * Sq + qr;
                const float* qv = q + qi * D;
                const float* gv = dO + qi * D;
                float dot = 0.0f, dov = 0.0f;
                for (int d = 0; d < D; ++d) { dot += qv[d] * kv[d]; dov += gv[d] * vv[d]; }
                const float p = expf(dot * scale - lse[qi]);
                const float ds = p * (dov - delta[qi]);
                for (int d = 0; d < D; ++d) {
                    gvv[d] += p * gv[d];
                    gk[d] += ds * qv[d] * scale;
                }
            }
        }
    }
    free(delta);
}

/*
 * RoPE on [BH, S, D] rows (rope.rs:68-96 fwd, :116-139 bwd).  pos = row
 * index s.  inv_freq_k = exp(k * (-2 ln(base) / D)), theta = pos * inv_freq.
 * style 0 = interleaved pairs (2k, 2k+1) as the reference; style 1 =
 * rotate-half pairs (k, k + D/2).  inverse != 0 applies the transposed
 * rotation (the reference backward).
 */
static inline void rope_row(const float* x, float* y, int pos, int D, float ln_base, int style,
                            int inverse) {
    const int half = D / 2;
    const float coef = -2.0f * ln_base / (float)D;
    for (int kk = 0; kk < half; ++kk) {
        const float inv_freq = expf((float)kk * coef);
        const float theta = (float)pos * inv_freq;
        const float c = cosf(theta);
        const float s = inverse ? -sinf(theta) : sinf(theta);
        const int i0 = style == 0 ? 2 * kk : kk;
        const int i1 = style == 0 ? 2 * kk + 1 : kk + half;
        const float a = x[i0], b = x[i1];
        y[i0] = a * c - b * s;
        y[i1] = a * s + b * c;
    }
}

ORC_EXPORT void orc_rope(const float* x, float* y, int BH, int S, int D, float ln_base,
                         int style, int inverse) {
    const long rows = (long)BH * S;
#pragma omp parallel for schedule(static)
    for (long r = 0; r < rows; ++r)
        rope_row(x + (size_t)r * D, y + (size_t)r * D, (int)(r % S), D, ln_base, style,
                 inverse);
}

/* [S, H*D] -> [H, S, D] per batch (transpose_heads.rs:59-70); pure copy. */
ORC_EXPORT void orc_transpose_heads(const void* src, void* dst, int B, int S, int H, int D,
                                    int elem_bytes) {
    const size_t row = (size_t)D * elem_bytes;
    const long rows = (long)B * S * H;
#pragma omp parallel for schedule(static)
    for (long r = 0; r < rows; ++r) {
        const long b = r / ((long)S * H), s = (r / H) % S, h = r % H;
        const char* from = (const char*)src + (size_t)r * row;
        char* to = (char*)dst + (((size_t)b * H + h) * S + s) * row;
        memcpy(to, from, row);
    }
}

/* [H, S, D] -> [S, H*D] per batch (transpose_heads.rs:86-95); pure copy. */
ORC_EXPORT void orc_merge_heads(const void* src, void* dst, int B, int S, int H, int D,
                                int elem_bytes) {
    const size_t row = (size_t)D * elem_bytes;
    const long rows = (long)B * S * H;
#pragma omp parallel for schedule(static)
    for (long r = 0; r < rows; ++r) {
        const long b = r / ((long)S * H), s = (r / H) % S, h = r % H;
        const char* from = (const char*)src + (((size_t)b * H + h) * S + s) * row;
        char* to = (char*)dst + (size_t)r * row;
        memcpy(to, from, row);
    }
}

/*
 * The attention layer's order (src/layers/attention.rs:97-123): transpose to
 * [B,H,S,D], then RoPE with pos = s.  inverse != 0 is the backward: inverse
 * rotation on [B,H,S,D], then merge back to [B,S,H,D].
 */
ORC_EXPORT void orc_rope_transpose(const float* x, float* y, int B, int S, int H, int D,
                                   float ln_base, int style, int inverse) {
    const size_t n = (size_t)B * S * H * D;
    float* tmp = (float*)malloc(sizeof(float) * (n ? n : 1));
    if (!inverse) {
        orc_transpose_heads(x, tmp, B, S, H, D, 4);
        orc_rope(tmp, y, B * H, S, D, ln_base, style, 0);
    } else {
        orc_rope(x, tmp, B * H, S, D, ln_base, style, 1);
        orc_merge_heads(tmp, y, B, S, H, D, 4);
    }
    free(tmp);
}

/*
 * Fused residual add + RMSNorm (fused_add_rmsnorm.rs:53-110): h = x + r,
 * rstd = rsqrt(sum(h^2) / N + eps), y = h * rstd * w.  r may be NULL
 * (plain RMSNorm); h_out may be NULL.
 */
ORC_EXPORT void orc_rmsnorm(const float* x, const float* r, const float* w, float* y,
                            float* h_out, int M, int N, float eps) {
#pragma omp parallel for schedule(static)
    for (long m = 0; m < M; ++m) {
        const float* xr = x + (size_t)m * N;
        const float* rr = r ? r + (size_t)m * N : NULL;
        float ss = 0.0f;
        for (int n = 0; n < N; ++n) {
            const float h = xr[n] + (rr ? rr[n] : 0.0f);
            if (h_out) h_out[(size_t)m * N + n] = h;
            ss += h * h;
        }
        const float rstd = 1.0f / sqrtf(ss * (1.0f / (float)N) + eps);
        for (int n = 0; n < N; ++n) {
            const float h = xr[n] + (rr ? rr[n] : 0.0f);
            y[(size_t)m * N + n] = h * rstd * w[n];
        }
    }
}

/* SwiGLU (swiglu.rs:56-95): z [M, 2*d_ff] = gate || up, out = silu(gate) * up. */
ORC_EXPORT void orc_swiglu(const float* z, float* out, int M, int d_ff) {
#pragma omp parallel for schedule(static)
    for (long m = 0; m < M; ++m)
        for (int n = 0; n < d_ff; ++n) {
            const float g = z[(size_t)m * 2 * d_ff + n];
            const float u = z[(size_t)m * 2 * d_ff + d_ff + n];
            const float sig = 1.0f / (1.0f + expf(-g));
            out[(size_t)m * d_ff + n] = g * sig * u;
        }
}
