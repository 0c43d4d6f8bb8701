// Declarations shared between the library's translation units.
#pragma once
#include "common.cuh"

namespace wk {

// ---------------------------------------------------------------- GEMV (gemv.cu)
enum Epi : int { EPI_STORE = 0, EPI_RESID = 1, EPI_QKV = 2, EPI_SWIGLU = 3, EPI_LOGITS = 4 };
constexpr int kMaxLogitCtas = 512;

struct GemvArgs {
    const uint8_t *w = nullptr;  // weight rows, raw GGUF bytes [N, K]
    int wtype = kQ8_0;
    int N = 0, K = 0;
    const void *x = nullptr;  // activations [M, ldx] (type T)
    long ldx = 0;
    int M = 0;                       // 1..8
    const float *norm_w = nullptr;   // RMSNorm prologue weight [K] (fp32) or null
    float eps = 1e-5f;
    int epi = EPI_STORE;
    void *out = nullptr;  // STORE / RESID / SWIGLU / QKV(q) / LOGITS(optional logits)
    long ldo = 0;
    const void *bias = nullptr;  // STORE: [N] (type T) or null
    const void *res = nullptr;   // RESID: residual [M, ldr]
    long ldr = 0;
    // QKV: features [0, nq) query, [nq, nq + nk) key, then value; RoPE on q/k
    int nq = 0, nk = 0, hd = 0;
    const float *freqs = nullptr;  // [ctx, hd] (cos, sin) pairs
    const int *pos = nullptr;      // [M] absolute position of each activation row
    const int *seq = nullptr;      // [M] sequence (block-table row) of each activation row
    void *kpool = nullptr, *vpool = nullptr;  // [pages][kv_heads][page][hd]
    const int *block_table = nullptr;          // [seqs][max_pages]
    int max_pages = 0, page = 0, kv_heads = 0;
    // SWIGLU: rows [0, F) up, [F, 2F) gate
    int F = 0;
    // LOGITS: argmax in the reference kernel's tie order
    float *part_val = nullptr;
    unsigned long long *part_key = nullptr;
    int *counter = nullptr;
    int *tokens = nullptr;
    int pack = 8;
    int *err = nullptr;
    int bulk = 1;  // set by gemv()
    int pdl = 1;   // launch with programmatic dependent launch
};

bool gemv_supported(int wtype, int act, int K);
void gemv(GemvArgs a, int act, cudaStream_t s);

// ---------------------------------------------------------------- ops.cu
template <typename T> void dequant_q8_0(T *out, const void *in, long nblocks, cudaStream_t s);
void embedding(void *out, const int *ids, const void *table, int n, int col, int dtype, int out_act, cudaStream_t s);
template <typename T> void rmsnorm(T *out, const T *in, const float *w, int rows, int C, float eps, cudaStream_t s);
template <typename T>
void rope(T *out, const T *in, const float *freqs, int batch, int row, int heads_per_row, int nrot, int HS, int pos0,
          cudaStream_t s);
template <typename T> void swiglu(T *out, const T *in, long rows, int C, cudaStream_t s);
template <typename T> void add(T *out, const T *a, const T *b, long n, cudaStream_t s);
template <typename T> void get_row(T *out, const T *in, int batch, int row, int col, int idx, cudaStream_t s);
template <typename T> void argmax(int *out, const T *in, int rows, int col, cudaStream_t s);

// ---------------------------------------------------------------- attention.cu
struct PagedKV {
    void *k = nullptr, *v = nullptr;  // [pages][kv_heads][page][hd] (type T)
    const int *block_table = nullptr;  // [seqs][max_pages]
    int max_pages = 0, page = 0, kv_heads = 0, hd = 0;
};
template <typename T>
void attention_paged(T *out, long out_rs, const T *q, long q_rs, const int *seq_of_row, const int *pos_of_row,
                     int nrows, int max_len, const PagedKV &c, int H, cudaStream_t s, bool pdl);
template <typename T>
void attention_qkv_rows(T *out, const T *qkv, int B, int Tn, int NH, int kvNH, int HS, cudaStream_t s);

// ---------------------------------------------------------------- matmul.cu
// out[M, N] = X[M, K] . W[N, K]^T (+bias), reference numerics; dispatches to the
// GEMV (M <= 8 per pass) or the generic kernel.
void matmul(void *out, const void *x, const void *w, const void *bias, int M, int K, int N, int wtype, int act,
            cudaStream_t s);
// Fill per-row metadata: seq[i] = i / n, pos[i] = pos0 + i % n.
void fill_row_meta(int *seq, int *pos, int rows, int n, int pos0, cudaStream_t s);
// Identity block table: bt[b][p] = b * pages + p.
void fill_block_table(int *bt, int batch, int pages, cudaStream_t s);

// ---------------------------------------------------------------- layers.cu
void layers_init();
void layers_fini();
void prefix_cache_forget(const void *ptr);
void prefix_cache_note_upload(void *dst, const void *src, size_t size);
void prefix_cache_note_write(void *dst, size_t size);
void prefix_cache_embedding(void *out, const int *ids, const void *embd, int batch, int row, int col, int dtype);

}  // namespace wk
