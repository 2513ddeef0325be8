/*
 * w8a8_oracle.c -- CPU restatement of vllm-turing's tensor-parallel W8A8 linear hot path, its int8 LM head (W8A16)
 * and its optional int8-compressed all-reduce (AR8).
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker: it is called by tests/, by __graft_entry__.smoke() and by
 * bench.py's cpu_baseline / `--impl reference` legs. The product path (vllm_turing_b200) never links, loads or calls
 * it; the CUDA library fails loudly instead of falling back to any CPU code.
 *
 * Parity pins: the quantisers, the dequant epilogue and the two-rank reduction are checked against golden vectors made
 * by the reference's own Python (vllm_turing/quantfuse.py quant_torch, imported from the reference tree) and by the
 * formulas its tests compute (tests/test_w8a8_mma.py:42-45, tests/test_quantfuse.py:45-48, tests/bench_devll.py:28-36);
 * the LM head's row quantiser and W8A16 arithmetic against the reference's vllm_turing/lmhead.py quantize_rows and its
 * large-M path run on the CPU; the AR8 format against the reference's own AR8 kernels rebuilt for the GPU (no golden
 * file: the GPU tests compare both bit for bit); see tests/golden/make_golden.py and tests/test_oracle.py.
 *
 * Every function names the reference file:line whose arithmetic it restates. Floating point follows the reference's
 * rounding points exactly (compile with -ffp-contract=off; fused multiply-adds are written out as fmaf where the
 * reference's nvcc build contracts them).
 *
 * dtype codes follow the reference's C ABI (vllm_turing/csrc/w8a8_gemv.cu:346): 0 = float16, 1 = bfloat16.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ---- 16-bit float helpers (round to nearest even) -------------------------------------------------------------- */
static inline float bf16_to_f(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}
static inline uint16_t f_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
static inline float f16_to_f(uint16_t h) {
    _Float16 x;
    memcpy(&x, &h, 2);
    return (float)x;
}
static inline uint16_t f_to_f16(float f) {
    _Float16 x = (_Float16)f; /* IEEE round to nearest even */
    uint16_t h;
    memcpy(&h, &x, 2);
    return h;
}
static inline float ld16(const uint16_t *p, long i, int dtype) { return dtype ? bf16_to_f(p[i]) : f16_to_f(p[i]); }
static inline uint16_t rnd16(float f, int dtype) { return dtype ? f_to_bf16(f) : f_to_f16(f); }

float orc_bf16_round(float f) { return bf16_to_f(f_to_bf16(f)); }

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void orc_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* ---- int8 GEMM, exact int32 accumulation ---------------------------------------------------------------------------
 * acc[m, n] = sum_k a[m, k] * w[n, k]; a [M, K] and w [N, K] row-major int8 (vLLM passes W as the transposed [K, N]
 * view of this row-major [N, K] tensor: vllm_turing/csrc/w8a8_gemv.cu:5, vllm_turing/w8a8.py:42).
 * Reference: the dp4a int32 dot products of w8a8_gemv_kernel (vllm_turing/csrc/w8a8_gemv.cu:53-71) and the int32
 * accumulator of the CUTLASS big GEMM (vllm_turing/csrc/w8a8_big.cu:40). int32 addition is associative, so the sum is
 * exact and independent of order as long as it does not overflow (|sum| <= K * 128 * 128 < 2^31 for K < 131072). */
void orc_gemm_s32(const int8_t *a, const int8_t *w, int32_t *acc, int M, int N, int K) {
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) {
        const int8_t *wr = w + (long)n * K;
        for (int m = 0; m < M; ++m) {
            const int8_t *ar = a + (long)m * K;
            int32_t s = 0;
            for (int k = 0; k < K; ++k) s += (int32_t)ar[k] * (int32_t)wr[k];
            acc[(long)m * N + n] = s;
        }
    }
}

/* ---- per-token x per-channel dequant epilogue ----------------------------------------------------------------------
 * out[m, n] = round_dtype(((float)acc * sa[m]) * sw[n] + bias[n]).
 * Reference: vllm_turing/csrc/w8a8_gemv.cu:87-91 (`(float) acc[r][m] * sa[sa_rows ? m : 0] * swn + b`, which nvcc
 * contracts to fma(acc * sa, sw, b)); sa_rows / sw_rows = 0 selects a per-tensor scale (w8a8.py:45). Without a
 * bias the expression is the plain product (fma with +0 differs only in the sign of an exact zero, which acc * sa * sw
 * with positive scales never produces except as +0). */
void orc_dequant(const int32_t *acc, const float *sa, const float *sw, const uint16_t *bias, uint16_t *out, int M,
                 int N, int sa_rows, int sw_rows, int dtype) {
#pragma omp parallel for schedule(static)
    for (int m = 0; m < M; ++m) {
        const float sam = sa[sa_rows ? m : 0];
        for (int n = 0; n < N; ++n) {
            const float t = (float)acc[(long)m * N + n] * sam;
            const float swn = sw[sw_rows ? n : 0];
            const float v = bias ? fmaf(t, swn, ld16(bias, n, dtype)) : t * swn;
            out[(long)m * N + n] = rnd16(v, dtype);
        }
    }
}

/* The prefill GEMM's epilogue order: out[m, n] = round_dtype(sa[m] * (sw[n] * (float)acc)).
 * Reference: the CUTLASS visitor tree of vllm_turing/csrc/w8a8_big.cu:26-35 (Compute0 = ScaleB * Acc, then
 * Compute1 = ScaleA * that, each a float32 multiply), which its test pins bitwise to vLLM's cutlass_scaled_mm
 * (tests/test_w8a8_big.py:49-54). */
void orc_dequant_big(const int32_t *acc, const float *sa, const float *sw, uint16_t *out, int M, int N, int dtype) {
#pragma omp parallel for schedule(static)
    for (int m = 0; m < M; ++m) {
        for (int n = 0; n < N; ++n) {
            const float t = sw[n] * (float)acc[(long)m * N + n];
            out[(long)m * N + n] = rnd16(sa[m] * t, dtype);
        }
    }
}

/* cutlass_scaled_mm semantics as the reference plugin serves them (vllm_turing/w8a8.py:108-117 -> gemv / mma). */
void orc_scaled_mm(const int8_t *a, const int8_t *w, const float *sa, const float *sw, const uint16_t *bias,
                   uint16_t *out, int M, int N, int K, int sa_rows, int sw_rows, int dtype) {
    int32_t *acc = (int32_t *)malloc(sizeof(int32_t) * (size_t)M * (size_t)N);
    if (!acc) return;
    orc_gemm_s32(a, w, acc, M, N, K);
    orc_dequant(acc, sa, sw, bias, out, M, N, sa_rows, sw_rows, dtype);
    free(acc);
}

/* ---- dynamic per-token symmetric int8 quantisation -----------------------------------------------------------------
 * Reference: vllm_turing/quantfuse.py:18-24 quant_torch: xf = float(x); absmax = max |xf| per row;
 * q = round_half_even(xf * (127 / absmax)).clamp(-128, 127); scale = absmax / 127. torch evaluates the scalar-over-
 * tensor `127.0 / absmax` as `absmax.reciprocal() * 127` (Tensor.__rtruediv__), i.e. two float32 roundings, and the
 * golden vectors of quant_torch pin exactly that (it decides ties such as x = absmax / 2 -> -63.5). An all-zero row
 * gives scale 0 and q = 0 (quant_torch yields 0 there; silu_quant.cu:57-58 states it as inv = 0). */
static void quant_row(const float *y, int8_t *q, float *scale, int N) {
    float amax = 0.0f;
    for (int n = 0; n < N; ++n) {
        const float v = fabsf(y[n]);
        amax = v > amax ? v : amax;
    }
    const float inv = amax > 0.0f ? (1.0f / amax) * 127.0f : 0.0f;
    *scale = amax / 127.0f;
    for (int n = 0; n < N; ++n) {
        float r = rintf(y[n] * inv); /* round half to even in the default rounding mode */
        r = r < -128.0f ? -128.0f : (r > 127.0f ? 127.0f : r);
        q[n] = (int8_t)r;
    }
}

void orc_quant_rows(const uint16_t *x, int8_t *q, float *scales, int M, int N, int dtype) {
#pragma omp parallel
    {
        float *row = (float *)malloc(sizeof(float) * (size_t)N);
#pragma omp for schedule(static)
        for (int m = 0; m < M; ++m) {
            for (int n = 0; n < N; ++n) row[n] = ld16(x, (long)m * N + n, dtype);
            quant_row(row, q + (long)m * N, scales + m, N);
        }
        free(row);
    }
}

/* ---- per-output-channel weight quantisation (checkpoint format) ----------------------------------------------------
 * Reference: scripts/w8a8_convert.py:165-166: scale = max(amax(|w|, row), 1e-12) / 127; q = round(w / scale)
 * clamped to [-128, 127] (a float32 division, round half to even). w float32 [N, K]. */
void orc_weight_quant(const float *w, int8_t *q, float *scale, int N, int K) {
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) {
        const float *wr = w + (long)n * K;
        float amax = 0.0f;
        for (int k = 0; k < K; ++k) {
            const float v = fabsf(wr[k]);
            amax = v > amax ? v : amax;
        }
        const float s = (amax < 1e-12f ? 1e-12f : amax) / 127.0f;
        scale[n] = s;
        for (int k = 0; k < K; ++k) {
            float r = rintf(wr[k] / s);
            r = r < -128.0f ? -128.0f : (r > 127.0f ? 127.0f : r);
            q[(long)n * K + k] = (int8_t)r;
        }
    }
}

/* ---- tensor-parallel all-reduce (sum) ------------------------------------------------------------------------------
 * out = round_dtype(sum over ranks r = 0..n-1 in rank order of float(part_r)), one rounding at the end.
 * Reference: the two-rank LL kernel adds in float32 and rounds once (vllm_turing/csrc/host_ar.cu:90-101:
 * __floats2bfloat162_rn(x.x + y.x, ...)); the oracle of its tests is (x0.float() + x1.float()).half()
 * (tests/bench_devll.py:28-36). For more than two ranks the build fixes the order 0, 1, ..., n-1 so every rank
 * computes the identical sum (float32 addition is not associative). */
void orc_all_reduce(const uint16_t *const *parts, int nranks, uint16_t *out, long n, int dtype) {
#pragma omp parallel for schedule(static)
    for (long i = 0; i < n; ++i) {
        float s = ld16(parts[0], i, dtype);
        for (int r = 1; r < nranks; ++r) s += ld16(parts[r], i, dtype);
        out[i] = rnd16(s, dtype);
    }
}

/* ---- residual add + RMSNorm + per-token int8 quantisation ----------------------------------------------------------
 * h = round_dtype(x + residual) (written back: the new residual, as vLLM's rms_norm_dynamic_per_token_quant updates
 * `res` in place, vllm_turing/tailoverlap.py:200-201); v = mean(float(h)^2); y = round_dtype(float(h) * rsqrt(v + eps)
 * * weight); (q, scale) = quant_torch(y).
 * Reference formula: tests/test_quantfuse.py:45-48 (`h = x + r`, `h.float() * torch.rsqrt(v + 1e-6) * (1.0 +
 * w.float())`) with the weight passed as the kernel takes it (the Gemma 1 + w is precomputed by the caller,
 * vllm_turing/tailoverlap.py:176-178); quantisation vllm_turing/quantfuse.py:18-24.
 * The mean of squares is accumulated in double here and rounded to float once (the reference's torch mean and the
 * CUDA tree sum both round differently in the last bit); rsqrt is the correctly rounded float of 1/sqrt.
 * `normed` (optional) receives y. */
void orc_add_rms_norm_quant(const uint16_t *x, uint16_t *residual, const uint16_t *weight, float eps, int8_t *q,
                            float *scales, uint16_t *normed, int M, int N, int dtype) {
#pragma omp parallel
    {
        float *h = (float *)malloc(sizeof(float) * (size_t)N);
        float *y = (float *)malloc(sizeof(float) * (size_t)N);
#pragma omp for schedule(static)
        for (int m = 0; m < M; ++m) {
            double ss = 0.0;
            for (int n = 0; n < N; ++n) {
                const long i = (long)m * N + n;
                const uint16_t hv = rnd16(ld16(x, i, dtype) + ld16(residual, i, dtype), dtype);
                residual[i] = hv;
                h[n] = ld16(&hv, 0, dtype);
                ss += (double)h[n] * (double)h[n];
            }
            const float v = (float)(ss / (double)N);
            const float rs = (float)(1.0 / sqrt((double)(v + eps)));
            for (int n = 0; n < N; ++n) {
                const float t = (h[n] * rs) * ld16(weight, n, dtype);
                const uint16_t yv = rnd16(t, dtype);
                y[n] = ld16(&yv, 0, dtype);
                if (normed) normed[(long)m * N + n] = yv;
            }
            quant_row(y, q + (long)m * N, scales + m, N);
        }
        free(h);
        free(y);
    }
}

/* ---- the whole row-parallel layer tail at tensor-parallel size n ---------------------------------------------------
 * per rank r: partial_r = scaled_mm(a_r, w_r, sa_r, sw_r) (its K-slice, vllm_turing/tailoverlap.py:147-150 `_proj`);
 * reduced = all_reduce(partial_0..n-1); residual, q, scales = add_rms_norm_quant(reduced, residual, weight).
 * Reference chain: tailoverlap.py:214-218 (plain tail: ar(_proj(...)) then mlp_partial's fused norm + quant,
 * tailoverlap.py:198-201). `reduced` (optional, [M, N]) receives the all-reduced sum. */
void orc_row_linear_tp(int nranks, const int8_t *const *a, const int8_t *const *w, const float *const *sa,
                       const float *const *sw, uint16_t *residual, const uint16_t *weight, float eps, int8_t *q,
                       float *scales, uint16_t *reduced, int M, int N, int K_local, int dtype) {
    uint16_t **parts = (uint16_t **)malloc(sizeof(uint16_t *) * (size_t)nranks);
    for (int r = 0; r < nranks; ++r) {
        parts[r] = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)M * (size_t)N);
        orc_scaled_mm(a[r], w[r], sa[r], sw[r], NULL, parts[r], M, N, K_local, 1, 1, dtype);
    }
    uint16_t *s = reduced ? reduced : (uint16_t *)malloc(sizeof(uint16_t) * (size_t)M * (size_t)N);
    orc_all_reduce((const uint16_t *const *)parts, nranks, s, (long)M * N, dtype);
    orc_add_rms_norm_quant(s, residual, weight, eps, q, scales, NULL, M, N, dtype);
    if (!reduced) free(s);
    for (int r = 0; r < nranks; ++r) free(parts[r]);
    free(parts);
}

/* ---- SiLU(gate) * up + per-row int8 quantisation (the MLP activation, next to the hot path) ------------------------
 * Reference: vllm_turing/csrc/silu_quant.cu:11-69: silu in float rounded to the 16-bit type, times up in the 16-bit
 * type (one rounding of the float product), then the dynamic quantisation of quantfuse.py:18-24. gu [M, 2I]. */
void orc_silu_mul_quant(const uint16_t *gu, int8_t *q, float *scales, int M, int I, int dtype) {
#pragma omp parallel
    {
        float *y = (float *)malloc(sizeof(float) * (size_t)I);
#pragma omp for schedule(static)
        for (int m = 0; m < M; ++m) {
            const long base = (long)m * 2 * I;
            for (int i = 0; i < I; ++i) {
                const float g = ld16(gu, base + i, dtype);
                const uint16_t sg = rnd16(g / (1.0f + expf(-g)), dtype);
                const uint16_t p = rnd16(ld16(&sg, 0, dtype) * ld16(gu, base + I + i, dtype), dtype);
                y[i] = ld16(&p, 0, dtype);
            }
            quant_row(y, q + (long)m * I, scales + m, I);
        }
        free(y);
    }
}

/* ---- all-gather -----------------------------------------------------------------------------------------------------
 * gathered = concat over ranks of each rank's payload (bytes). Reference: vllm_turing/csrc/dma_ag.cu:41-47 (rank r's
 * payload occupies bytes [r*m, (r+1)*m) of `gathered`). */
void orc_all_gather(const uint8_t *const *payloads, int nranks, uint8_t *gathered, long m) {
    for (int r = 0; r < nranks; ++r) memcpy(gathered + (long)r * m, payloads[r], (size_t)m);
}

/* ---- LM head: per-row weight quantisation -------------------------------------------------------------------------
 * Reference: vllm_turing/lmhead.py:52-61 (quantize_rows): sc = max(amax(|w|, row), 1e-12) / 127 in float32,
 * q = round(w / sc) (half to even) clamped to [-128, 127]. w float32 [N, K] (the fp16 / bf16 head widened).
 * The reference runs it on the GPU after loading (lmhead.py:125-128), where torch evaluates a tensor divided by a
 * Python scalar as a multiplication by the float32 reciprocal: sc = amax * fl(1 / 127) (recip = 1). On the CPU torch
 * divides (recip = 0). The division w / sc is a true float32 division on both. */
void orc_lmhead_quant(const float *w, int8_t *q, float *scale, int N, int K, int recip) {
    const float inv127 = 1.0f / 127.0f;
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) {
        const float *wr = w + (long)n * K;
        float amax = 0.0f;
        for (int k = 0; k < K; ++k) {
            const float v = fabsf(wr[k]);
            amax = v > amax ? v : amax;
        }
        const float a = amax < 1e-12f ? 1e-12f : amax;
        const float s = recip ? a * inv127 : a / 127.0f;
        scale[n] = s;
        for (int k = 0; k < K; ++k) {
            float r = rintf(wr[k] / s);
            r = r < -128.0f ? -128.0f : (r > 127.0f ? 127.0f : r);
            q[(long)n * K + k] = (int8_t)r;
        }
    }
}

/* ---- LM head: W8A16 GEMM -----------------------------------------------------------------------------------------
 * out[m, n] = round_dtype(fma(acc, s[n], bias[n])) with acc = sum_k x[m, k] * w[n, k]; x [M, K] 16-bit bits, w [N, K]
 * int8, s [N] float32, bias [N] 16-bit bits or NULL.
 * Reference: vllm_turing/csrc/w8a16_gemv.cu:64-106 (fp32 FMAs of an int8 weight and a 16-bit activation per lane,
 * a shuffle tree, then `acc * s[ns] + b`, which nvcc contracts to one fma). Every product is exact in fp32; the
 * reference's fp32 sum depends on its lane order, so the oracle takes the sum in double (the value every fp32 order
 * approximates) and reports mag[m, n] = sum_k |x w|, which bounds the summation error of any fp32 order by
 * about K * 2^-24 * mag. acc and mag may be NULL. */
void orc_w8a16(const uint16_t *x, const int8_t *w, const float *s, const uint16_t *bias, uint16_t *out, double *acc,
               double *mag, int M, int N, int K, int dtype) {
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) {
        const int8_t *wr = w + (long)n * K;
        const float b = bias ? ld16(bias, n, dtype) : 0.0f;
        for (int m = 0; m < M; ++m) {
            const uint16_t *xr = x + (long)m * K;
            double sum = 0.0, mg = 0.0;
            for (int k = 0; k < K; ++k) {
                const double p = (double)wr[k] * (double)ld16(xr, k, dtype);
                sum += p;
                mg += fabs(p);
            }
            out[(long)m * N + n] = rnd16(fmaf((float)sum, s[n], b), dtype);
            if (acc) acc[(long)m * N + n] = sum;
            if (mag) mag[(long)m * N + n] = mg;
        }
    }
}

/* ---- AR8: the compressed all-reduce (optional, lossy) -------------------------------------------------------------
 * Reference: vllm_turing/csrc/host_ar.cu:133-201. Packed block of n fp16 values (n % 128 == 0): n int8, then n / 128
 * fp16 scales. Per 128-element group: amax = max |x|; sc = fp16(amax / 127) (float32 division, round to nearest
 * even); inv = sc > 0 ? 1 / (float)sc : 0; q = clamp(rint(x * inv), -127, 127) (host_ar.cu:138-160). */
void orc_ar8_quant(const uint16_t *x, uint8_t *packed, long n) {
    int8_t *q = (int8_t *)packed;
    uint16_t *sc = (uint16_t *)(packed + n);
    const long ng = n / 128;
#pragma omp parallel for schedule(static)
    for (long g = 0; g < ng; ++g) {
        float amax = 0.0f;
        for (int j = 0; j < 128; ++j) {
            const float v = fabsf(f16_to_f(x[g * 128 + j]));
            amax = v > amax ? v : amax;
        }
        const uint16_t sh = f_to_f16(amax / 127.0f);
        const float s = f16_to_f(sh);
        const float inv = s > 0.0f ? 1.0f / s : 0.0f;
        for (int j = 0; j < 128; ++j) {
            float r = rintf(f16_to_f(x[g * 128 + j]) * inv);
            r = r < -127.0f ? -127.0f : (r > 127.0f ? 127.0f : r);
            q[g * 128 + j] = (int8_t)r;
        }
        sc[g] = sh;
    }
}

/* out[i] = fp16(sum over ranks r = 0..world-1 in order of q_r[i] * sc_r[i / 128]) with float32 additions; gathered =
 * world packed blocks of n + n / 64 bytes. Reference: ar8_dequant_sum_kernel (host_ar.cu:163-180), two ranks:
 * `u * a0 + w * a1` -- both products are exact in float32, so its one rounding is the oracle's. */
void orc_ar8_dequant_sum(const uint8_t *gathered, uint16_t *out, long n, int world) {
    const long blk = n + n / 64;
#pragma omp parallel for schedule(static)
    for (long i = 0; i < n; ++i) {
        float acc = 0.0f;
        for (int r = 0; r < world; ++r) {
            const int8_t *q = (const int8_t *)(gathered + r * blk);
            const uint16_t *sc = (const uint16_t *)(gathered + r * blk + n);
            const float p = (float)q[i] * f16_to_f(sc[i / 128]);
            acc = r == 0 ? p : acc + p;
        }
        out[i] = f_to_f16(acc);
    }
}
