/*
 * wukong.h -- the C ABI of the B200 (sm_100a) wukong op library.
 *
 * Drop-in for the reference's cuda.h (liuy/wukong, cuda.h:1-28): the same 28
 * declarations with the same argument meaning, called by llm/array.go through
 * cgo.  Pointers are device pointers unless named host; activations use T =
 * float / bf16 / half selected by the weight dtype exactly as the reference
 * does (half for F16 and every quantised dtype).  Errors abort the process with
 * a message, as the reference's panic macro does.
 */
#ifndef WUKONG_B200_H
#define WUKONG_B200_H
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* cuda.h:1  (cuda.cu:1017-1049)  select device `idx`, create the library stream */
void cuda_init(int idx);
/* cuda.h:2  (cuda.cu:1051-1057)  release the library's device state */
void cuda_fini(void);
/* cuda.h:3  (cuda.cu:1060-1065)  stream-ordered device allocation */
void* cuda_malloc(size_t size);
/* cuda.h:4  (cuda.cu:1077-1082)  device -> host copy; synchronises the stream */
void cuda_to_host(void* dst, void* src, size_t size);
/* cuda.h:5  (cuda.cu:1072-1075)  host -> device copy, asynchronous */
void cuda_to_device(void* dst, void* src, size_t size);
/* cuda.h:6  (cuda.cu:1067-1070)  stream-ordered free */
void cuda_free(void* ptr);
/* cuda.h:7  (cuda.cu:1095-1111)  out[row, oc] = inp[row, column] . weight[oc, column]^T (+bias);
 * weight dtype F32 / F16 / BF16 / Q8_0 (Q8_0: half activations) */
void cuda_matmul(void *out, const void *inp, const void *weight, const void *bias, int row, int column, int oc, int dtype);
/* cuda.h:8  (cuda.cu:1120-1126)  fp32 row softmax */
void cuda_softmax(void* output, void* input, int row, int col);
/* cuda.h:9  (cuda.cu:1182-1185)  causal MHA on fp32 [batch, row, 3 NH HS] rows */
void cuda_mh_sdpa(void *out, const void *inp, int batch, int row, int NH, int HS);
/* cuda.h:10 (cuda.cu:1139-1145)  causal GQA on fp32 [batch, row, (qNH + 2 kvNH) HS] rows */
void cuda_gq_sdpa(void *out, const void *inp, int batch, int row, int qNH, int kvNH, int HS);
/* cuda.h:11 (cuda.cu:1197-1203)  causal MQA (kvNH = 1) */
void cuda_mq_sdpa(void *out, const void *inp, int batch, int row, int qNH, int HS);
/* cuda.h:12 (cuda.cu:1156-1159)  fp32 RMSNorm with fp32 weight */
void cuda_rmsnorm(void *out, const void *inp, const void *weight, int row, int col, float eps);
/* cuda.h:13 (cuda.cu:1164-1167)  fp32 SwiGLU: out = up * silu(gate), input rows [up | gate] */
void cuda_swiglu(void *out, const void *inp, int batch, int row, int col);
/* cuda.h:14 (cuda.cu:1217-1220)  fp32 RoPE on the Q and K heads of fused QKV rows */
void cuda_rope_qkv(void *out, const void *inp, const void *freqs, int batch, int row, int NH, int kvNH, int HS);
/* cuda.h:15 (declared, never defined by the reference)  fp32 RoPE on [batch, row, NH, HS] */
void cuda_rope(void *out, const void *inp, const void *freqs, int batch, int row, int NH, int HS);
/* cuda.h:16 (cuda.cu:1232-1255)  row gather by int32 id; Q8_0 tables are dequantised to half */
void cuda_embedding(void* out, const void *inp, const void *embd, int batch, int row, int col, int dtype);
/* cuda.h:17 (cuda.cu:1267-1275)  row concatenation */
void cuda_cat(void *out, const void *a, const void *b, int arow, int brow, int col, int dtype);
/* cuda.h:18 (cuda.cu:1286-1293)  fp32 element-wise a / b */
void cuda_div(void *out, const void *a, const void *b, int row, int col);
/* cuda.h:19 (cuda.cu:1305-1308)  Q8_0 -> fp32, bit-exact */
void cuda_dequantize(void *out, const void *inp, int row, int col, int type);
/* cuda.h:20 (cuda.cu:1319-1322)  fp32 element-wise a + b */
void cuda_add(void* out, const void* a, const void* b, int row, int col);
/* cuda.h:21 (cuda.cu:1324-1338, :902-926)  attention sublayer with residual, in place when out == embeds */
void cuda_group_query_attention(void *out, const void *embeds, const void *freqs, const void *norm_weight, const void *qkv_weight, const void *out_weight, int batch, int row, int NH, int kvNH, int HS, float eps, int dtype);
/* cuda.h:22 (cuda.cu:1351-1354)  fp32 K/V replication to [batch, row, 3 qNH HS] */
void cuda_repeat_qkv(void *out, const void *inp, int batch, int row, int qNH, int kvNH, int HS);
/* cuda.h:23 (cuda.cu:1384-1400, :928-945)  SwiGLU FFN sublayer with residual */
void cuda_feed_forward(void *out, const void *attn, const void *norm_weight, const void *fc_weight, const void *out_weight, int batch, int row, int col, int ffl, float eps, int dtype);
/* cuda.h:24 (cuda.cu:1366-1369)  fp32 row `idx` (negative: from the end) of each batch */
void cuda_get_row(void *out, const void *inp, int batch, int row, int col, int idx);
/* cuda.h:25 (cuda.cu:1402-1414, :975-981)  logits of the last row: [batch, wsize] in T */
void cuda_classify(void *out, void *ff, const void *norm_weight, const void *out_weight, int batch, int row, int col, int wsize, float eps, int dtype);
/* cuda.h:26 (cuda.cu:1379-1382)  fp32 row argmax -> int32, the reference kernel's tie order */
void cuda_argmax(void *out, const void *inp, int row, int col);
/* cuda.h:27 (cuda.cu:1416-1428, :983-990)  greedy next token ids (int32 [batch]) */
void cuda_predict(void *out, void *ff, const void *norm_weight, const void *out_weight, int batch, int row, int col, int wsize, float eps, int dtype);

#ifdef __cplusplus
}
#endif
#endif
