/*
 * wukong_ext.h -- extended C API of the B200 wukong library: a native Llama-3
 * decode engine with a paged KV cache, batched greedy decode and CUDA-graph
 * replay.  The reference has no counterpart; its Go runtime drives the same
 * computation through cuda.h (llm/llama.go:117-154 per step, re-running the
 * whole sequence).  This API is what bench.py and C hosts use to run the hot
 * path without re-prefill.
 *
 * Conventions: all tensor arguments are device pointers, borrowed (the caller
 * keeps them alive); weights are raw GGUF bytes in the llama.go layout (fused
 * q|k|v rows, fused up|gate rows).  Functions return 0 on success and a
 * negative code on error; wk_last_error() describes the last error.
 * cuda_init() must have been called first (the engine runs on its stream).
 */
#ifndef WUKONG_B200_EXT_H
#define WUKONG_B200_EXT_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct wk_model wk_model;

typedef struct {
    int n_layers, d_model, n_heads, n_kv_heads, head_dim, ffn, vocab;
    float eps;
    int wtype;       /* dtype of the linear layers (GGML id: 1 F16, 2 Q4_0, 8 Q8_0, 30 BF16) */
    int out_wtype;   /* dtype of output.weight */
    int embd_wtype;  /* dtype of token_embd.weight (0 F32, 1 F16, 2 Q4_0, 8 Q8_0, 30 BF16) */
} wk_config;

const char *wk_last_error(void);

wk_model *wk_model_create(const wk_config *cfg);
void wk_model_destroy(wk_model *m);
/* per layer l: attn_norm [d] f32, qkv [(H + 2 Hk) D, d], o [d, d], ffn_norm [d] f32,
 * fc [2 F, d] (up rows then gate rows), down [d, F] */
int wk_model_set_layer(wk_model *m, int l, const void *attn_norm, const void *qkv, const void *o,
                       const void *ffn_norm, const void *fc, const void *down);
/* token_embd [V, d], output_norm [d] f32, output [V, d], freqs [ctx, D] f32 (cos, sin pairs) */
int wk_model_set_head(wk_model *m, const void *token_embd, const void *output_norm, const void *output,
                      const void *freqs, int freqs_ctx);
/* paged KV cache for up to max_batch sequences of up to max_ctx tokens each */
int wk_model_alloc_cache(wk_model *m, int max_batch, int max_ctx);

/* Prefill: batch sequences, each with n prompt tokens (device int32 [batch, n]),
 * positions 0..n-1; writes the greedy next token of each sequence to
 * tokens_out (device int32 [batch]) and arms the decode state. */
int wk_model_prefill(wk_model *m, const int *ids, int batch, int n, int *tokens_out);
/* One greedy decode step for the armed batch: consumes the last tokens,
 * appends one position, writes the next tokens to the internal token buffer.
 * The first call captures the step into a CUDA graph; later calls replay it. */
int wk_model_decode_step(wk_model *m);
/* Continuous batching (no counterpart in the reference, whose Go loop decodes
 * one sequence at a time, llm/model.go:116-178): sequences of different
 * lengths join and leave the decode batch while it runs.  Each lives in a
 * slot 0..max_batch-1 of the paged cache.  wk_model_add_seqs prefills count
 * new sequences (ids: device int32, the prompts back to back; lens: host int
 * [count]) into the lowest free slots (host slots_out [count]), appends them as
 * the last rows of the batch and writes their first generated tokens there.
 * wk_model_remove_seq drops a slot's sequence (the last row takes its row).
 * wk_model_rows writes the slot of every decode row (host int [batch]) and
 * returns the batch size; wk_model_tokens / wk_model_next_ids are in row
 * order.  A decode step advances every row by one position; the batch's
 * graph is re-captured after the batch changes.  Not with tensor parallelism. */
int wk_model_add_seqs(wk_model *m, const int *ids, const int *lens, int count, int *slots_out);
int wk_model_remove_seq(wk_model *m, int slot);
int wk_model_rows(const wk_model *m, int *slots);
/* device [batch, vocab] logits (activation dtype) of the latest step's last
 * rows while sampling is on (wk_model_set_sampling), else null */
const void *wk_model_logits(const wk_model *m);
/* device int32 [batch]: tokens produced by the latest prefill / decode step */
const int *wk_model_tokens(const wk_model *m);
/* device int32 [batch]: input tokens of the next decode step (writable) */
int *wk_model_next_ids(wk_model *m);
/* number of this library's kernel launches in one decode step */
int wk_model_step_launches(const wk_model *m);
/* current sequence length (positions used) */
int wk_model_position(const wk_model *m);
/* Roll every armed sequence back to n positions (1 <= n <= current length):
 * the next decode step writes position n again, overwriting the cached K/V
 * from there on.  The next input ids (wk_model_next_ids) are left as they are;
 * the caller sets them.  Used to discard speculative or timed continuations. */
int wk_model_truncate(wk_model *m, int n);

/* Sampling instead of greedy argmax (the reference's predict is greedy and
 * leaves sampling as a TODO, cuda.cu:988): temperature > 0 turns it on for
 * the model's prefill and decode steps, temperature <= 0 back to greedy.  The
 * candidates are the min(top_k, 256) largest logits (top_k <= 0: 256), equal
 * values ordered by smaller index; top_p in (0, 1) keeps the shortest prefix
 * of them whose probability reaches top_p.  The draw of the token at
 * position p + 1 of sequence b uses the counter-based uniform of (seed, p, b),
 * so a run is reproducible.  Call after wk_model_alloc_cache; not with
 * tensor parallelism.  Returns 0 or -1. */
int wk_model_set_sampling(wk_model *m, float temperature, int top_k, float top_p, unsigned long long seed);
/* The same sampling over logits rows already on the device ([rows, vocab] of
 * dtype F16, BF16 or F32, e.g. from cuda_classify), every row with RNG step
 * `step`: device int32 tokens[rows]. */
int wk_sample_logits(int *tokens, const void *logits, int rows, int vocab, int dtype, float temperature, int top_k,
                     float top_p, unsigned long long seed, long long step);

/* The engine's decode attention on its own: out[rows][n_heads * head_dim] for
 * query rows q[rows][n_heads * head_dim], row r the newest token of sequence
 * seq[r] at position pos[r] (keys 0..pos[r]), over the paged cache kpool /
 * vpool [pages][kv_heads][64][head_dim] with block_table[seqs][max_pages];
 * max_len bounds every pos[r] + 1.  dtype F16 or BF16.  The kernel is the
 * one decode steps use (a cluster of CTAs per (row, KV head); the one-CTA
 * kernel with WUKONG_SPLIT_ATTN=0 or WUKONG_CLUSTER_ATTN=0).  No counterpart
 * in the reference, whose attention recomputes K and V from the rows.
 * Returns 0 or -1. */
int wk_attention_decode(void *out, const void *q, const void *kpool, const void *vpool, const int *block_table,
                        int max_pages, const int *seq, const int *pos, int rows, int max_len, int n_heads,
                        int kv_heads, int head_dim, int dtype);

/* Synthetic weights, bit-identical to the CPU oracle's generator:
 * Irwin-Hall(4) normal(0, stdv) samples of a counter-based hash. */
int wk_fill_random_q8_0(void *dst, long rows, int cols, uint64_t seed, float stdv);
/* The same samples quantised to GGUF Q4_0 (d = largest-magnitude value / -8,
 * nibble = min(15, (int)(x / d + 8.5))). */
int wk_fill_random_q4_0(void *dst, long rows, int cols, uint64_t seed, float stdv);
int wk_fill_random_f16(void *dst, long n, uint64_t seed, float stdv);
int wk_fill_const_f32(void *dst, long n, float value);

/* Direct GEMV entry (decode matmul): out[M, N] = x[M, K] . W[N, K]^T, M <= 8,
 * half activations for F16/Q8_0 weights.  For benchmarking the op alone. */
int wk_gemv(void *out, const void *x, const void *w, int M, int K, int N, int wtype);

/* library stream (cudaStream_t) so hosts can order their own work */
void *wk_stream(void);

/* Tensor parallelism inside one node, one process per GPU (no counterpart in
 * the reference, which runs on one device): column-parallel q|k|v and up|gate,
 * row-parallel o and down with an fp32 all-reduce after each, vocabulary-
 * parallel logits with a winner exchange; NCCL is loaded at run time.
 * Rank r of `world`: wk_tp_unique_id on one rank, share the 128 bytes, then
 * wk_tp_init(r, world, id) on every rank after cuda_init.  A model made for TP
 * holds the rank's shard: wk_config's n_heads, n_kv_heads, ffn and vocab are
 * the per-rank counts (global / world); qkv = [q heads r*H..][k heads r*Hk..]
 * [v heads r*Hk..] rows, o = the K-columns of those q heads, fc = [up rows
 * r*F..][gate rows r*F..], down = the K-columns r*F.., output = vocabulary rows
 * r*V..; embeddings and norms are whole.  Call wk_model_set_tp(m, 1) before
 * wk_model_alloc_cache.  Every rank runs the same calls in the same order. */
int wk_tp_unique_id(void *id);
int wk_tp_init(int rank, int world, const void *id);
void wk_tp_fini(void);
int wk_tp_rank(void);
int wk_tp_world(void);
/* 1 when the ranks exchange decode-sized partials through each other's memory
 * (one fused all-reduce + residual launch over NVLink), 0 when they use NCCL
 * (WUKONG_TP_P2P=0, or a rank could not map the others' buffers) */
int wk_tp_p2p(void);
int wk_model_set_tp(wk_model *m, int enable);
/* The exchange of wk_tp_p2p on this one GPU, for testing the failure path:
 * ranks 1..world-1 are emulated by buffers on this device.  publish = 1 writes
 * their partial sums and flags first, so the exchange completes and its sum is
 * checked; publish = 0 leaves them unwritten, so every CTA's bounded wait runs
 * out (after WUKONG_WAIT_LIMIT_MS, read at cuda_init; default 1000) and
 * records code 40 in the device error word.  Returns the error word after the
 * launch (0: completed), -2 for a wrong sum, -1 for a setup error.  Does not
 * need wk_tp_init. */
int wk_tp_exchange_selftest(int world, int publish);
/* The decode GEMV whose epilogue exchanges its partial tiles (the o / down
 * layers of tensor-parallel decode) on this one GPU with ranks 1..world-1
 * emulated by buffers that hold published partials of 0.25 q: checks that
 * x = T(x + T(own partial + sum of the others)) element for element against
 * the same GEMV's partial sums.  Q8_0 [N, K] weights, M rows (<= 8).  Returns
 * 0, the device error word, or -2 with the first wrong element in
 * wk_last_error(). */
int wk_tp_gemv_selftest(int world, int N, int K, int M);
/* The device error word: the code of the first bounded device wait that gave
 * up since it was last cleared (0: none), after synchronising the library
 * stream; clear = 1 resets it.  cuda_to_host ends the process when it is set,
 * and wk_model_prefill / wk_model_decode_step refuse to launch (return -1). */
int wk_device_error(int clear);

/* No counterpart in the reference.  cuda_predict without device allocation,
 * for hosts that cannot call cudaMalloc at that point: a process that has
 * given all free HBM to its own KV-cache pool, or a latency-critical loop in
 * which cudaMalloc / cudaFree would synchronise the device.  Same arguments
 * and result as cuda_predict (greedy next-token ids, int32 [batch], of the
 * last row of each of the batch sequences in ff) for F16, BF16 and Q8_0
 * output weights, same kernel.  Its scratch is a fixed 393,472-byte array
 * inside the library (every GPU that loads the library holds it until exit),
 * so a call takes at most 64 sequences and col <= 32768; larger or unsupported
 * sizes return -1 with the reason in wk_last_error().  CUDA errors inside the
 * GEMV launch end the process with a message, as cuda_predict's do.  All calls
 * share that array: calls that overlap on the GPU race; calls on the library
 * stream do not.  The first call on a device looks up the array's address
 * (cached until cuda_fini); make it before any stream capture.  Returns 0 on
 * success. */
int wk_predict_noalloc(int *out, const void *ff, const void *norm_weight, const void *out_weight, int batch,
                       int row, int col, int wsize, float eps, int dtype);

/* Decode-step timeline (no counterpart in the reference; diagnostic build
 * libwukong_timeline.so from `python -m wukong_b200.build --timeline`, where
 * every GEMV and decode-attention launch records per CTA %globaltimer at its
 * start, after griddepcontrol.wait, at phase marks and at its end; the default
 * library returns -1 from the first two).  wk_timeline_init(slots, blocks)
 * allocates [slots][blocks] records and restarts the count; wk_timeline_read
 * copies info [slots][4] (kind, N, K, CTAs) and stamps [slots][blocks][9]
 * (start, wait return, end, phases 0..5) and returns the launches recorded
 * (launch i in slot i mod slots).  wk_timeline_resolution_ns: the smallest
 * step of %globaltimer one thread observes. */
int wk_timeline_init(int slots, int blocks);
int wk_timeline_read(int *info, unsigned long long *stamps);
long long wk_timeline_resolution_ns(void);

#ifdef __cplusplus
}
#endif
#endif
