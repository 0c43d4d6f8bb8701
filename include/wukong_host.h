/*
 * wukong_host.h -- host-side mirror of the reference's Go runtime for the hot
 * path (llm/llama.go Setup/Predict, llm/model.go Generate), written against a
 * table of cuda.h entry points so that it drives any library exporting that ABI.
 */
#ifndef WUKONG_B200_HOST_H
#define WUKONG_B200_HOST_H
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* cuda.h entry points used by the Go hot path (llm/array.go:373-778) */
typedef struct {
    void (*cuda_init)(int);
    void (*cuda_fini)(void);
    void *(*cuda_malloc)(size_t);
    void (*cuda_to_host)(void *, void *, size_t);
    void (*cuda_to_device)(void *, void *, size_t);
    void (*cuda_free)(void *);
    void (*cuda_cat)(void *, const void *, const void *, int, int, int, int);
    void (*cuda_embedding)(void *, const void *, const void *, int, int, int, int);
    void (*cuda_group_query_attention)(void *, const void *, const void *, const void *, const void *, const void *,
                                       int, int, int, int, int, float, int);
    void (*cuda_feed_forward)(void *, const void *, const void *, const void *, const void *, int, int, int, int,
                              float, int);
    void (*cuda_predict)(void *, void *, const void *, const void *, int, int, int, int, float, int);
} wk_abi;

/* model hyper-parameters (llm/model.go:23-36) and GGUF dtypes */
typedef struct {
    int n_layers, d_model, n_heads, n_kv_heads, head_dim, ffn, vocab, ctx;
    float eps, rope_theta;
    int wtype, out_wtype, embd_wtype;
} wk_host_config;

/* per-layer GGUF tensors (device pointers, unfused as in the file) */
typedef struct {
    const void *attn_norm, *q, *k, *v, *o, *ffn_norm, *up, *gate, *down;
} wk_host_layer;

typedef struct wk_host_llama wk_host_llama;

const char *wk_host_last_error(void);
/* resolve the cuda.h entry points from a dlopen() handle */
int wk_abi_bind(wk_abi *table, void *dl_handle);
void wk_host_make_freqs(float *out, const float *factor, int HS, int ctx, float theta);
wk_host_llama *wk_host_llama_create(const wk_abi *abi, const wk_host_config *cfg);
void wk_host_llama_destroy(wk_host_llama *h);
/* llama.go:69-115 (output == NULL ties the logits weight to token_embd) */
int wk_host_llama_setup(wk_host_llama *h, const wk_host_layer *layers, const void *token_embd,
                        const void *output_norm, const void *output, const float *rope_factor);
/* llama.go:117-154: ids host [batch, seqs] -> next ids host [batch] */
int wk_host_llama_predict(wk_host_llama *h, const int *ids, int batch, int seqs, int *out);
/* model.go:116-178 greedy loop (no tokenizer, no stop token): steps predictions */
int wk_host_llama_generate(wk_host_llama *h, const int *prompt, int n_prompt, int steps, int *out_tokens);

#ifdef __cplusplus
}
#endif
#endif
