// Host-side mirror of the reference's Go runtime above the C ABI:
//   llama.go:54-67   makeFreqsTensor     -> host_make_freqs
//   llama.go:69-115  Llama3Handler.Setup -> wk_host_llama_setup (q|k|v and
//                                           up|gate fusion through cuda_cat)
//   llama.go:117-154 Llama3Handler.Predict -> wk_host_llama_predict
//   model.go:116-178 Model.Generate      -> wk_host_llama_generate (greedy)
// Every device operation goes through a table of cuda.h entry points, bound by
// dlsym to a library handle: this library, or any other build of the same ABI
// (the reference's own cuda.cu compiled for sm_100a), so one host loop drives
// both.  Same call sequence, buffer ownership and argument values as the Go
// code: ids are uploaded with cuda_to_device every step, outputs are
// cuda_malloc'ed and freed, the predicted ids come back with cuda_to_host.
#include <dlfcn.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "wukong_host.h"

namespace {

#define WK_SYMS(X)                \
    X(cuda_init)                  \
    X(cuda_fini)                  \
    X(cuda_malloc)                \
    X(cuda_to_host)               \
    X(cuda_to_device)             \
    X(cuda_free)                  \
    X(cuda_cat)                   \
    X(cuda_embedding)             \
    X(cuda_group_query_attention) \
    X(cuda_feed_forward)          \
    X(cuda_predict)

char g_host_err[512];

}  // namespace

struct wk_host_llama {
    wk_abi abi;
    wk_host_config cfg;
    // device tensors (owned through the bound ABI)
    void **qkv, **fc;        // fused per layer (llama.go:80-112)
    const void **attn_norm, **o, **ffn_norm, **down;
    const void *token_embd, *output_norm, *output;
    void *freqs;  // [ctx, D] fp32
};

extern "C" {

const char *wk_host_last_error(void) { return g_host_err; }

int wk_abi_bind(wk_abi *t, void *handle) {
    memset(t, 0, sizeof(*t));
#define BIND(n)                                                                           \
    t->n = (decltype(t->n))dlsym(handle, #n);                                             \
    if (!t->n) {                                                                          \
        snprintf(g_host_err, sizeof(g_host_err), "symbol %s not found: %s", #n, dlerror()); \
        return -1;                                                                        \
    }
    WK_SYMS(BIND)
#undef BIND
    return 0;
}

// llama.go:54-67
void wk_host_make_freqs(float *out, const float *factor, int HS, int ctx, float theta) {
    for (int i = 0; i < HS / 2; ++i) {
        float freq = 1.0f / (float)pow((double)theta, (double)(2 * i) / (double)HS);
        freq /= factor ? factor[i] : 1.0f;
        for (int j = 0; j < ctx; ++j) {
            float angle = (float)j * freq;
            out[(long)j * HS + 2 * i] = (float)cos((double)angle);
            out[(long)j * HS + 2 * i + 1] = (float)sin((double)angle);
        }
    }
}

static size_t tensor_bytes(long rows, long cols, int dtype) {
    switch (dtype) {
    case 0: return (size_t)rows * cols * 4;
    case 1:
    case 30: return (size_t)rows * cols * 2;
    case 8: return (size_t)rows * (cols / 32) * 34;
    default: return 0;
    }
}

wk_host_llama *wk_host_llama_create(const wk_abi *abi, const wk_host_config *cfg) {
    wk_host_llama *h = (wk_host_llama *)calloc(1, sizeof(wk_host_llama));
    h->abi = *abi;
    h->cfg = *cfg;
    const int L = cfg->n_layers;
    h->qkv = (void **)calloc(L, sizeof(void *));
    h->fc = (void **)calloc(L, sizeof(void *));
    h->attn_norm = (const void **)calloc(L, sizeof(void *));
    h->o = (const void **)calloc(L, sizeof(void *));
    h->ffn_norm = (const void **)calloc(L, sizeof(void *));
    h->down = (const void **)calloc(L, sizeof(void *));
    return h;
}

void wk_host_llama_destroy(wk_host_llama *h) {
    if (!h) return;
    for (int l = 0; l < h->cfg.n_layers; ++l) {
        if (h->qkv[l]) h->abi.cuda_free(h->qkv[l]);
        if (h->fc[l]) h->abi.cuda_free(h->fc[l]);
    }
    if (h->freqs) h->abi.cuda_free(h->freqs);
    free(h->qkv);
    free(h->fc);
    free(h->attn_norm);
    free(h->o);
    free(h->ffn_norm);
    free(h->down);
    free(h);
}

// llama.go:69-115: builds the RoPE table and fuses q|k|v and up|gate with
// cuda_cat.  Weights are device tensors the caller keeps alive (the Go code
// frees the unfused ones; the caller may do so after this returns).
int wk_host_llama_setup(wk_host_llama *h, const wk_host_layer *layers, const void *token_embd,
                        const void *output_norm, const void *output, const float *rope_factor) {
    const wk_host_config &c = h->cfg;
    const int d = c.d_model, D = c.head_dim, H = c.n_heads, Hk = c.n_kv_heads;
    float *f = (float *)malloc(sizeof(float) * (size_t)c.ctx * D);
    wk_host_make_freqs(f, rope_factor, D, c.ctx, c.rope_theta);
    const size_t fbytes = sizeof(float) * (size_t)c.ctx * D;
    h->freqs = h->abi.cuda_malloc(fbytes);
    h->abi.cuda_to_device(h->freqs, f, fbytes);
    free(f);
    h->token_embd = token_embd;
    h->output_norm = output_norm;
    h->output = output ? output : token_embd;  // llama.go:75-78 ties output to token_embd
    for (int l = 0; l < c.n_layers; ++l) {
        const wk_host_layer &w = layers[l];
        void *qk = h->abi.cuda_malloc(tensor_bytes((long)(H + Hk) * D, d, c.wtype));
        h->abi.cuda_cat(qk, w.q, w.k, H * D, Hk * D, d, c.wtype);
        h->qkv[l] = h->abi.cuda_malloc(tensor_bytes((long)(H + 2 * Hk) * D, d, c.wtype));
        h->abi.cuda_cat(h->qkv[l], qk, w.v, (H + Hk) * D, Hk * D, d, c.wtype);
        h->abi.cuda_free(qk);
        h->fc[l] = h->abi.cuda_malloc(tensor_bytes(2L * c.ffn, d, c.wtype));
        h->abi.cuda_cat(h->fc[l], w.up, w.gate, c.ffn, c.ffn, d, c.wtype);
        h->attn_norm[l] = w.attn_norm;
        h->o[l] = w.o;
        h->ffn_norm[l] = w.ffn_norm;
        h->down[l] = w.down;
    }
    return 0;
}

// llama.go:117-154 with the cudaRunner calls of array.go:659-778.
int wk_host_llama_predict(wk_host_llama *h, const int *ids, int batch, int seqs, int *out) {
    const wk_host_config &c = h->cfg;
    const wk_abi &a = h->abi;
    const int d = c.d_model;
    if (seqs > c.ctx) {
        snprintf(g_host_err, sizeof(g_host_err), "sequence %d exceeds context %d", seqs, c.ctx);
        return -1;
    }
    // MakeTensor(Shape{batch, seqs}, flat)
    void *d_ids = a.cuda_malloc(sizeof(int) * (size_t)batch * seqs);
    a.cuda_to_device(d_ids, (void *)ids, sizeof(int) * (size_t)batch * seqs);
    // Embedding (array.go:659-688): quantised tables produce half rows
    const int et = c.embd_wtype;
    const size_t es = (et == 0) ? 4 : 2;
    void *embeds = a.cuda_malloc(es * (size_t)batch * seqs * d);
    a.cuda_embedding(embeds, d_ids, h->token_embd, batch, seqs, d, et);
    // freqs.RowSlice(0, seqs) is a view of the table start
    for (int l = 0; l < c.n_layers; ++l) {
        a.cuda_group_query_attention(embeds, embeds, h->freqs, h->attn_norm[l], h->qkv[l], h->o[l], batch, seqs,
                                     c.n_heads, c.n_kv_heads, c.head_dim, c.eps, c.wtype);
        a.cuda_feed_forward(embeds, embeds, h->ffn_norm[l], h->fc[l], h->down[l], batch, seqs, d, c.ffn, c.eps,
                            c.wtype);
    }
    // Predict (array.go:763-778)
    void *d_out = a.cuda_malloc(sizeof(int) * batch);
    a.cuda_predict(d_out, embeds, h->output_norm, h->output, batch, seqs, d, c.vocab, c.eps, c.out_wtype);
    a.cuda_to_host(out, d_out, sizeof(int) * batch);
    a.cuda_free(d_out);
    a.cuda_free(embeds);
    a.cuda_free(d_ids);
    return 0;
}

// model.go:116-178 without the tokenizer/printing: greedy steps appending the
// predicted id to the sequence and re-running Predict on the whole sequence.
int wk_host_llama_generate(wk_host_llama *h, const int *prompt, int n_prompt, int steps, int *out_tokens) {
    int *ids = (int *)malloc(sizeof(int) * (size_t)(n_prompt + steps));
    memcpy(ids, prompt, sizeof(int) * n_prompt);
    int len = n_prompt;
    for (int s = 0; s < steps; ++s) {
        int next;
        if (wk_host_llama_predict(h, ids, 1, len, &next)) {
            free(ids);
            return -1;
        }
        out_tokens[s] = next;
        ids[len++] = next;
    }
    free(ids);
    return 0;
}

}  // extern "C"
