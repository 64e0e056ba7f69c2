/*
 * oracle.c — CPU restatement of the reference's algorithms for the GPT-2 decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This is the checker the CUDA kernels are compared against
 * (tests/, __graft_entry__.smoke, and bench.py's cpu_baseline / --impl reference legs).
 * Nothing in the product library links or calls it.
 *
 * Pinned against the reference itself: oracle/build_ref.sh compiles the reference's own
 * CPU attention harness (tests/test_paged_attention.cu:138-179) and its K13/K14 CUDA
 * kernels from their sources into oracle/_ref/; tests/test_oracle_pins.py checks this file
 * against the harness (bit-exact) and against numpy quantize_per_row fixtures
 * (tests/golden/, made by tests/golden/make_golden.py from python/export_gpt2.py:10-40).
 *
 * Every function follows a reference file:line given in its comment, keeping the
 * reference's summation order and float types so results are bit-comparable.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <stdlib.h>
#include <float.h>

#ifdef _OPENMP
#include <omp.h>
#endif

static inline float bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline float kv_at(const void* cache, int kv_dtype, size_t idx) {
    if (kv_dtype == 0) return ((const float*)cache)[idx];
    return bf16_to_f32(((const uint16_t*)cache)[idx]);
}

/*
 * Decode attention for one query token per sequence over a paged, ragged KV cache.
 *
 * Restates gqa_cpu_reference (reference tests/test_paged_attention.cu:138-179) for the
 * decode case the K13 test exercises (N_q = 1, non-causal: tests/test_decode_attention.cu:100-110):
 *   scale = 1/sqrtf(d); kv head = hq / (H_q/H_kv);
 *   s_j = (sum_k q[k]*K[j][k]) * scale;  max-subtracted expf;  divide by the sum;  O = P.V
 * with K/V row j of sequence b at ((bt[b][j/bs]*bs + j%bs)*H_kv + hkv)*d (the K13 address,
 * kernels/decode/13_decode_attn.cuh:97) and ctx_b = context_lens[b] keys. A zero-length
 * context gives O = 0 (the intended result of the reference's reduce, 13_decode_attn.cu:48-52).
 * kv_dtype 1 = bf16 cache, upcast exactly to fp32.
 */
void oracle_decode_attn(int B, int H_q, int H_kv, int d, const float* Q, const void* k_cache,
                        const void* v_cache, int kv_dtype, const int* block_table,
                        const int* context_lens, int block_size, int num_blocks_per_seq, float* O,
                        int nthreads) {
    const float scale = 1.0f / sqrtf((float)d);
    const int group = H_q / H_kv;
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel for collapse(2) schedule(dynamic) num_threads(nthreads)
#endif
    for (int b = 0; b < B; ++b) {
        for (int hq = 0; hq < H_q; ++hq) {
            const int hkv = hq / group;
            const int ctx = context_lens[b];
            const float* q = Q + ((size_t)b * H_q + hq) * d;
            float* o = O + ((size_t)b * H_q + hq) * d;
            if (ctx <= 0) {
                for (int dd = 0; dd < d; ++dd) o[dd] = 0.0f;
                continue;
            }
            float* scores = (float*)malloc(sizeof(float) * (size_t)ctx);
            size_t* rows = (size_t*)malloc(sizeof(size_t) * (size_t)ctx);
            float max_s = -FLT_MAX;
            for (int j = 0; j < ctx; ++j) {
                const int phys = block_table[(size_t)b * num_blocks_per_seq + j / block_size];
                rows[j] = (((size_t)phys * block_size + (size_t)(j % block_size)) * H_kv + hkv) * d;
                float sum = 0.0f;
                for (int kk = 0; kk < d; ++kk) sum += q[kk] * kv_at(k_cache, kv_dtype, rows[j] + kk);
                scores[j] = sum * scale;
                if (scores[j] > max_s) max_s = scores[j];
            }
            float sum_exp = 0.0f;
            for (int j = 0; j < ctx; ++j) {
                scores[j] = expf(scores[j] - max_s);
                sum_exp += scores[j];
            }
            for (int j = 0; j < ctx; ++j) scores[j] /= sum_exp;
            for (int dd = 0; dd < d; ++dd) {
                float sum = 0.0f;
                for (int j = 0; j < ctx; ++j) sum += scores[j] * kv_at(v_cache, kv_dtype, rows[j] + dd);
                o[dd] = sum;
            }
            free(scores);
            free(rows);
        }
    }
}

/*
 * Per-row symmetric quantisation (reference kernels/quantization/14_int8_gemm.cu:22-58 and
 * python/export_gpt2.py:22-38): amax = max |x|; scale = amax>0 ? amax/127 : 1;
 * inv = 1/scale; q = clamp(rint(x*inv), -128, 127) with round-half-even; pack byte j of
 * int32 i = element 4i+j.
 */
void oracle_quantize(int rows, int cols, const float* in, int32_t* out, float* scales) {
    for (int r = 0; r < rows; ++r) {
        const float* x = in + (size_t)r * cols;
        float amax = 0.0f;
        for (int c = 0; c < cols; ++c) {
            const float v = fabsf(x[c]);
            if (v > amax) amax = v;
        }
        const float scale = amax > 0.0f ? amax / 127.0f : 1.0f;
        const float inv = 1.0f / scale;
        scales[r] = scale;
        for (int i = 0; i < cols / 4; ++i) {
            uint32_t packed = 0;
            for (int j = 0; j < 4; ++j) {
                const float prod = x[4 * i + j] * inv;
                float q = rintf(prod);
                if (q < -128.0f) q = -128.0f;
                if (q > 127.0f) q = 127.0f;
                packed |= (uint32_t)(uint8_t)(int8_t)(int)q << (8 * j);
            }
            out[(size_t)r * (cols / 4) + i] = (int32_t)packed;
        }
    }
}

/* Scalar int32 GEMM: C[m,n] = sum_k A[m,k]*B[n,k] over int8 bytes of the packed operands
 * (the contraction of int8_gemm_dp4a_kernel, reference kernels/quantization/14_int8_gemm.cu:96-140). */
void oracle_int8_gemm_s32(int M, int N, int K, const int32_t* A, const int32_t* BT, int32_t* C,
                          int nthreads) {
    const int8_t* a8 = (const int8_t*)A;
    const int8_t* b8 = (const int8_t*)BT;
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel for schedule(static) num_threads(nthreads)
#endif
    for (int m = 0; m < M; ++m) {
        const int8_t* ar = a8 + (size_t)m * K;
        for (int n = 0; n < N; ++n) {
            const int8_t* br = b8 + (size_t)n * K;
            int32_t acc = 0;
            for (int k = 0; k < K; ++k) acc += (int32_t)ar[k] * (int32_t)br[k];
            C[(size_t)m * N + n] = acc;
        }
    }
}

/* Epilogue of the reference K14 (kernels/quantization/14_int8_gemm.cu:154-167):
 *   v = float(acc)*sA[m]*sB[n]; +bias; GELU-tanh; +residual.
 * nvcc contracts `t*sB + bias` and `v + 0.044715*x3` into fused multiply-adds in the
 * reference build, so the same fmaf calls appear here. tanhf is the host libm's. */
static inline float epi_apply(int epi, int32_t acc, float sa, float sb, float bias, float res) {
    const float t = (float)acc * sa;
    if (epi == 0) return t * sb;
    float v = fmaf(t, sb, bias);
    if (epi == 1) return v;
    if (epi == 2) {
        const float x3 = (v * v) * v;
        const float inner = 0.7978845608f * fmaf(0.044715f, x3, v);
        return (0.5f * v) * (1.0f + tanhf(inner));
    }
    return v + res;
}

void oracle_int8_gemm(int M, int N, int K, const int32_t* A, const int32_t* BT, const float* sA,
                      const float* sB, const float* bias, const float* residual, float* C, int epi,
                      int nthreads) {
    int32_t* acc = (int32_t*)malloc(sizeof(int32_t) * (size_t)M * N);
    oracle_int8_gemm_s32(M, N, K, A, BT, acc, nthreads);
    for (int m = 0; m < M; ++m)
        for (int n = 0; n < N; ++n) {
            const size_t i = (size_t)m * N + n;
            C[i] = epi_apply(epi, acc[i], sA[m], sB[n], epi ? bias[n] : 0.0f,
                             epi == 3 ? residual[i] : 0.0f);
        }
    free(acc);
}

/* Epilogue alone over given int32 accumulators (used to compare dequantised outputs). */
void oracle_epilogue(int M, int N, const int32_t* acc, const float* sA, const float* sB,
                     const float* bias, const float* residual, float* C, int epi) {
    for (int m = 0; m < M; ++m)
        for (int n = 0; n < N; ++n) {
            const size_t i = (size_t)m * N + n;
            C[i] = epi_apply(epi, acc[i], sA[m], sB[n], epi ? bias[n] : 0.0f,
                             epi == 3 ? residual[i] : 0.0f);
        }
}

int oracle_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* LayerNorm (reference kernels/layernorm/15_layernorm_residual.cu:59-103): mean = sum/cols,
 * var = sumsq/cols - mean^2, inv = 1/sqrt(var + eps) (the GPU uses rsqrtf),
 * y = gamma*(x-mean)*inv + beta, the last step fused as in the reference build. */
void oracle_layernorm(int rows, int cols, const float* x, const float* gamma, const float* beta, float eps,
                      float* y) {
    /* Sums in the reference kernel's order (kernels/layernorm/15_layernorm_residual.cu:59-103,
       256 threads): thread t accumulates columns t, t+256, ... (sum of squares fused, as the
       GPU build contracts it), then partial[t] += partial[t+s] for s = 128, 64, ..., 1. The
       reference's rsqrtf is replaced by a correctly rounded 1/sqrt (they differ by at most a
       couple of ulp), so rows agree with the GPU to about 1e-7 relative, not bit for bit. */
    float ps[256], pq[256];
    for (int r = 0; r < rows; ++r) {
        const float* xr = x + (size_t)r * cols;
        for (int t = 0; t < 256; ++t) {
            float s = 0.0f, q = 0.0f;
            for (int c = t; c < cols; c += 256) {
                s += xr[c];
                q = fmaf(xr[c], xr[c], q);
            }
            ps[t] = s;
            pq[t] = q;
        }
        for (int st = 128; st > 0; st >>= 1)
            for (int t = 0; t < st; ++t) {
                ps[t] += ps[t + st];
                pq[t] += pq[t + st];
            }
        const float mean = ps[0] / (float)cols;
        const float var = fmaf(-mean, mean, pq[0] / (float)cols);
        const float inv = (float)(1.0 / sqrt((double)(var + eps)));
        for (int c = 0; c < cols; ++c) y[(size_t)r * cols + c] = fmaf(gamma[c] * (xr[c] - mean), inv, beta[c]);
    }
}

/* Tied fp32 vocab projection (reference src/gpt2_engine.cu:391-403): logits[b,v] = sum_k h[b,k]*wte[v,k]. */
void oracle_vocab_proj(int B, int V, int d, const float* h, const float* wte, float* logits, int nthreads) {
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel for schedule(static) num_threads(nthreads)
#endif
    for (int v = 0; v < V; ++v)
        for (int b = 0; b < B; ++b) {
            float sum = 0.0f;
            /* sequential in k with a fused multiply-add per term, as the reference's kernel
               compiles on the GPU */
            for (int k = 0; k < d; ++k) sum = fmaf(h[(size_t)b * d + k], wte[(size_t)v * d + k], sum);
            logits[(size_t)b * V + v] = sum;
        }
}
