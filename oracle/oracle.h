/*
 * CPU oracle for the wukong hot path -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain C/C++ restatement of the semantics of the reference's CUDA op library
 * (cuda.cu of liuy/wukong), used by tests/ and by bench.py's CPU-baseline leg as
 * the checker.  Nothing in wukong_b200/ links or calls this library.
 *
 * Conventions
 *  - Activations are passed as float32 arrays whose values lie on the grid of the
 *    activation type `act` (ORC_F32, ORC_F16, ORC_BF16).  Every function rounds
 *    its stored results to that grid at the same points where the reference
 *    stores a T-typed buffer (cuda.cu instantiates T = half for F16 and for every
 *    quantised weight type, cuda.cu:1324-1338).
 *  - Weights are raw GGUF bytes with their GGML dtype (ORC_F32, ORC_F16,
 *    ORC_BF16, ORC_Q8_0).
 *  - Accumulation is fp32 (as cuBLAS with CUBLAS_COMPUTE_32F, cuda.cu:294-297).
 */
#pragma once
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORC_F32 = 0, ORC_F16 = 1, ORC_Q4_0 = 2, ORC_Q8_0 = 8, ORC_BF16 = 30 };

/* element helpers */
float orc_round(int act, float x);
void orc_round_array(int act, float *x, size_t n);
void orc_f16_to_f32(const uint16_t *src, float *dst, size_t n);
void orc_f32_to_f16(const float *src, uint16_t *dst, size_t n);
void orc_bf16_to_f32(const uint16_t *src, float *dst, size_t n);
void orc_f32_to_bf16(const float *src, uint16_t *dst, size_t n);

/* cuda.cu:389-421 -- Q8_0 dequantisation; out_half != 0 rounds to fp16 */
void orc_dequant_q8_0(float *out, const uint8_t *blocks, int rows, int cols, int out_half);

/* cuda.cu:1095-1111 + :270-341 -- out[M,N] = X[M,K] . W[N,K]^T (+bias) */
void orc_matmul(float *out, const float *x, const void *w, const float *bias,
                int M, int K, int N, int wtype, int act);

void orc_rmsnorm(float *out, const float *x, const float *w, int rows, int C, float eps, int act); /* :533-601 */
void orc_rope_qkv(float *qkv, const float *freqs, int batch, int row, int pos0,
                  int NH, int kvNH, int HS, int act);                                 /* :207-236 */
void orc_rope(float *x, const float *freqs, int batch, int row, int NH, int HS, int act);
void orc_swiglu(float *out, const float *inp, int rows, int C, int act);               /* :176-205 */
void orc_add(float *out, const float *a, const float *b, size_t n, int act);           /* :423-435 */
void orc_div(float *out, const float *a, const float *b, size_t n);                    /* :379-387 */
void orc_softmax(float *out, const float *inp, int rows, int cols);                    /* :86-158 */
/* :437-467 repeat + :767-852 sdpa, causal, scale 1/sqrt(HS), GQA groups */
void orc_gqa_sdpa(float *out, const float *qkv, int batch, int row, int NH, int kvNH, int HS, int act);
/* :469-478 */
void orc_get_row(float *out, const float *inp, int batch, int row, int col, int idx);
/* :480-531, with the kernel's exact tie order; pack = 16 / sizeof(T) */
void orc_argmax(int *out, const float *inp, int rows, int cols, int pack);
void orc_gen_q4_0(uint8_t *out, int rows, int cols, uint64_t seed, float stdv);
void orc_quantize_q4_0(uint8_t *out, const float *x, int rows, int cols);
void orc_dequant_q4_0(float *out, const uint8_t *blocks, int rows, int cols, int out_half);
void orc_sample(int *out, float *u_out, const float *logits, int rows, int V, float temperature, int top_k,
                float top_p, uint64_t seed, const int64_t *steps);
/* :238-252 + :1232-1255; out in act grid (Q8_0 -> fp16) */
void orc_embedding(float *out, const int *ids, const void *table, int n, int col, int dtype);

/* Layer drivers with a KV cache (cuda.cu:902-945, :975-990).
 * x: residual [B, n, d] for the n new rows at absolute positions pos0..pos0+n-1.
 * kcache/vcache: [B, kvNH, cap, HS] (act grid); rows [0, pos0) must hold the
 * keys/values of earlier positions.  pos0 = 0, n = T is the reference's full
 * recompute; per-row results do not depend on pos0. */
void orc_gqa_layer(float *x, const float *freqs, const float *norm_w, const void *qkv_w,
                   const void *out_w, int B, int n, int pos0, int NH, int kvNH, int HS,
                   float eps, int wtype, int act, float *kcache, float *vcache, int cap);
void orc_ffn_layer(float *x, const float *norm_w, const void *fc_w, const void *down_w,
                   int B, int n, int d, int F, float eps, int wtype, int act);
/* logits for the last row of each batch: out_logits [B, V] (act grid), tokens [B] */
void orc_classify(float *logits, const float *x, const float *norm_w, const void *w,
                  int B, int T, int d, int V, float eps, int wtype, int act);

/* Synthetic weights: counter-based normal(0, std) samples (Irwin-Hall of 4
 * 16-bit uniforms, integer exact) -- identical bytes on CPU and GPU. */
void orc_gen_normal(float *dst, size_t n, uint64_t seed, float stdv);
void orc_gen_q8_0(uint8_t *dst, int rows, int cols, uint64_t seed, float stdv);
void orc_gen_f16(uint16_t *dst, size_t n, uint64_t seed, float stdv);
/* GGUF-style Q8_0 quantiser: d = max|w|/127 (fp32), q = roundf(w/d), scale stored fp16 */
void orc_quantize_q8_0(uint8_t *dst, const float *src, int rows, int cols);

/* llama.go:54-67 makeFreqsTensor: [ctx, HS] (cos, sin interleaved) */
void orc_make_freqs(float *out, const float *factor, int HS, int ctx, float theta);

int orc_num_threads(void);
/* F32-weight matmuls with TF32 (round-to-nearest) inputs, as cuBLASLt's
 * COMPUTE_32F_FAST_TF32 (cuda.cu:1046-1048); default off (exact fp32). */
void orc_set_f32_tf32(int on);
void orc_set_threads(int n);

#ifdef __cplusplus
}
#endif
