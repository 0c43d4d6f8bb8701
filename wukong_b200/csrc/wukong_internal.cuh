// Declarations shared between the library's translation units.
#pragma once
#include <cuda.h>  // CUtensorMap (types only; the encoder is fetched at run time)

#include "common.cuh"

namespace wk {

// ---------------------------------------------------------------- TMA (tma.cu)
// Tensor maps are encoded on the host with cuTensorMapEncodeTiled, resolved via
// cudaGetDriverEntryPoint so that the library links without libcuda.
bool encode_map_2d(CUtensorMap *m, const void *base, CUtensorMapDataType dt, uint64_t inner, uint64_t outer,
                   uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle);
// Cached map over a weight matrix viewed as [N rows][row_bytes / 2] uint16 with
// boxes of `box_inner` uint16 x `box_rows` rows (null if the rows are not TMA-able).
const CUtensorMap *weight_map(const void *w, long rows, long row_bytes, int box_inner, int box_rows);
void forget_weight_maps(const void *w);

// ---------------------------------------------------------------- GEMV (gemv.cu)
// PARTIAL: fp32 partial sums (no rounding) of a K-slice, reduced across ranks later.
// ARESID: tensor-parallel row-parallel layer in decode: the tile's fp32
// partial sums are exchanged with every rank through peer memory and the
// residual is added to their sum, x = T(x + T(sum over ranks)), in the GEMV's
// own epilogue (no separate all-reduce launch).
enum Epi : int {
    EPI_STORE = 0,
    EPI_RESID = 1,
    EPI_QKV = 2,
    EPI_SWIGLU = 3,
    EPI_LOGITS = 4,
    EPI_PARTIAL = 5,
    EPI_ARESID = 6
};
constexpr int kMaxLogitCtas = 512;

// ---------------------------------------------------------------- peer exchange of tensor parallelism
// Every rank exports one buffer that all ranks map (tp.cu); its layout:
constexpr int kTpMaxTiles = 512;  // 16-row output tiles of a row-parallel layer (d <= 8192)
constexpr size_t kXArFlags = 0;                              // [2 parities][16 CTAs] u64: all-reduce kernel
constexpr size_t kXWinFlags = 256;                           // [2 parities] u64: logits winners
constexpr size_t kXArPay = 512;                              // [2][kXArSlot] fp32 all-reduce payload
constexpr size_t kXArSlot = 256 * 1024;
constexpr size_t kXWinPay = kXArPay + 2 * kXArSlot;          // [2][kXWinSlot] winners: keys u64 [B], values f32 [B]
constexpr size_t kXWinSlot = 4096;
// Decode exchanges of the GEMV epilogues are pushed, not pulled: a rank
// stores each value together with the call's epoch in one 8-byte word
// (value bits low, epoch high) into every peer's buffer, and a receiver polls
// its own words until the epoch matches -- one NVLink write per value and no
// system-scope fence or separate flag (single-copy atomic 8-byte stores).
constexpr int kTpMaxWorld = 8;
constexpr size_t kXTileLL = kXWinPay + 2 * kXWinSlot;  // [2][kTpMaxTiles][kTpMaxWorld src][128] u64
constexpr size_t kXWinLL = kXTileLL + 2 * (size_t)kTpMaxTiles * kTpMaxWorld * 128 * 8;  // [2][src][8 rows][4] u64
constexpr size_t kXBytes = kXWinLL + 2 * (size_t)kTpMaxWorld * 8 * 4 * 8;

// What a kernel needs to exchange with the other ranks (device pointers).
struct TpLink {
    uint8_t *const *peers = nullptr;           // [world] exchange buffers of all ranks (own at [rank])
    int rank = 0, world = 1;
    unsigned long long *tile_epoch = nullptr;  // [kTpMaxTiles] ARESID calls that published each tile (own)
    unsigned long long *win_epoch = nullptr;   // [1] logits winner exchanges so far (own)
    unsigned long long limit_ns = 1000000000ull;
};
// The exchange of this process's ranks, or false when the ranks use NCCL.
bool tp_link(TpLink *link);

struct GemvArgs {
    CUtensorMap wmap;  // weight tiles (64-byte aligned first member; set by gemv())
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
    long col_off = 0;   // vocabulary shard: global column of local row 0
    int n_total = 0;    // vocabulary size of the whole row (0: N)
    float *best_val = nullptr;             // optional per-row winner (value, key) instead of / beside tokens
    unsigned long long *best_key = nullptr;
    const void *pf = nullptr;  // weights of a later kernel to prefetch into L2
    long pf_bytes = 0;
    int *err = nullptr;
    int bulk = 1;  // set by gemv(): 1 when the weight tiles stream by TMA
    int pdl = 1;   // launch with programmatic dependent launch
    int warp_tile_min = 1 << 30;  // set by gemv() from g_rt.warp_tile_min
    // ARESID, and LOGITS of a vocabulary shard with tokens set: the exchange
    // with the other ranks (tp.world > 1)
    TpLink tp;
    // 1: the epilogue's side inputs (residual; positions, block table and RoPE
    // table) were written two or more launches earlier in a stream whose kernels
    // all let their dependents start only after their own griddepcontrol.wait,
    // so they are complete when this kernel starts and are read before its wait
    int pre = 0;
};
static_assert(alignof(GemvArgs) >= 64, "the tensor map must stay 64-byte aligned");

bool gemv_supported(int wtype, int act, int K);
// Linear layers with many 16-row tiles (the logits of Llama-sized models) give
// each warp whole tiles: all K-chunks accumulate in one warp, in K order, and
// the warp applies the epilogue itself.  Fewer tiles are split over the 8 warps
// of a CTA by K-chunk and reduced in shared memory.  The rule depends only on
// the layer shape and the process-wide threshold (g_rt.warp_tile_min), so the
// per-op GEMV and the persistent decode kernel round identically.
__host__ __device__ inline bool warp_tiles(int epi, int ntiles, int min_tiles) {
    return (epi == EPI_SWIGLU || epi == EPI_LOGITS) && ntiles >= min_tiles;
}
void gemv(GemvArgs a, int act, cudaStream_t s);

// ---------------------------------------------------------------- tcgen05 GEMM (gemm_tc.cu)
// Same epilogues as the GEMV (no LOGITS), any M, 16-byte aligned rows.
struct GemmArgs {
    CUtensorMap wmap;  // weights (set by gemm_tc)
    CUtensorMap xmap;  // activations (set by gemm_tc)
    const uint8_t *w = nullptr;
    int wtype = kQ8_0;
    int N = 0, K = 0;
    const void *x = nullptr;
    long ldx = 0;
    int M = 0;
    int epi = EPI_STORE;
    void *out = nullptr;
    long ldo = 0;
    const void *bias = nullptr;
    const void *res = nullptr;
    long ldr = 0;
    int nq = 0, nk = 0, hd = 0;
    const float *freqs = nullptr;
    const int *pos = nullptr;
    const int *seq = nullptr;
    void *kpool = nullptr, *vpool = nullptr;
    const int *block_table = nullptr;
    int max_pages = 0, page = 0, kv_heads = 0;
    int F = 0;
    int *err = nullptr;
    int pdl = 1;
    int vec = 0;  // set by gemm_tc(): the epilogue stores 8 outputs (16 bytes) per access
    int ksplit = 1;              // set by gemm_tc(): K slices (gridDim.z)
    float *ws = nullptr;         // split-K partial tiles [tiles][ksplit][128][BN]
    int *ws_counter = nullptr;   // [tiles] arrivals, zero between launches
};
bool gemm_tc_supported(int wtype, int act, int K, int N, int epi, int F);
void gemm_tc(GemmArgs a, int act, cudaStream_t s);
// Minimum activation rows for which the tcgen05 GEMM replaces the GEMV
// (measured, 8192 x 2048 Q8_0, M = 16: 19.6 us on tcgen05, 24.3 us as two 8-row GEMV passes).
constexpr int kTcMinRows = 16;

// ---------------------------------------------------------------- sampling.cu
// Temperature / top-k / top-p sampling of one token per logits row.  The RNG
// step of row b is pos[b * pos_stride + pos_off] when pos is set, else step.
struct SampleArgs {
    float temperature = 1.f;
    int top_k = 0;
    float top_p = 1.f;
    unsigned long long seed = 0;
    long long step = 0;
    const int *pos = nullptr;
    long pos_stride = 1;
    int pos_off = 0;
};
void sample_rows(int *tokens, const void *logits, long ld, int rows, int V, int act, const SampleArgs &p,
                 cudaStream_t s);

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
// Scratch of split-K decode attention (sized by its owner; counter zeroed once).
struct AttnSplitWs {
    void *scores = nullptr;     // [max_rows][max_kv_heads][8][lpad] (type T)
    float *mpart = nullptr;     // [max_rows][max_kv_heads][max_splits][16]: 8 maxima, 8 sums of exp(s - max)
    float *opart = nullptr;     // [max_rows][max_kv_heads][max_splits][8][head_dim]
    int *counter = nullptr;     // [max_rows][max_kv_heads], zero between launches (P.V launch)
    int *counter_a = nullptr;   // the same for the scores launch
    float *minv = nullptr;      // [max_rows][max_kv_heads][8][2] row max and 1 / softmax sum per head
    int max_rows = 0, max_kv_heads = 0, max_splits = 0, lpad = 0;
};
// Returns the number of kernel launches.
// early: every row is the newest token of its sequence and older pages were
// written by earlier launches (decode), so they may be fetched before the
// programmatic-dependent-launch wait.
template <typename T>
int attention_paged(T *out, long out_rs, const T *q, long q_rs, const int *seq_of_row, const int *pos_of_row,
                     int nrows, int max_len, const PagedKV &c, int H, cudaStream_t s, bool pdl,
                     const void *pf = nullptr, long pf_bytes = 0, bool early = false,
                     const AttnSplitWs *ws = nullptr);
template <typename T>
void attention_qkv_rows(T *out, const T *qkv, int B, int Tn, int NH, int kvNH, int HS, cudaStream_t s);
// Prefill rows: n positions P..P+n-1 of each of `batch` sequences (q row b n + i
// is position P + i) over the paged cache, flash-style on tensor cores with
// the reference's rounding points.  Returns 1 (launches), or -1 when the
// shapes are not supported (16-bit K/V, 64-token pages, head_dim 64 / 128,
// 1, 2, 4 or 8 query heads per KV head) and attention_paged must be used.
template <typename T>
int attention_prefill_paged(T *out, long out_rs, const T *q, long q_rs, int batch, int n, int P, const PagedKV &c,
                            int H, cudaStream_t s);

// ---------------------------------------------------------------- matmul.cu
// out[M, N] = X[M, K] . W[N, K]^T (+bias), reference numerics; dispatches to the
// GEMV (M <= 8 per pass) or the generic kernel.
void matmul(void *out, const void *x, const void *w, const void *bias, int M, int K, int N, int wtype, int act,
            cudaStream_t s);
// One linear layer with a fused epilogue over `rows` activation rows described
// by `g` (g.M is ignored).  rows >= kTcMinRows run on the tcgen05 GEMM (an
// RMSNorm prologue becomes a separate pass into norm_scratch, [rows, K]);
// fewer rows run as GEMV passes of <= 8 rows (pf only on the first pass).
// Returns the number of kernel launches.
int linear(const GemvArgs &g, int rows, int act, cudaStream_t s, void *norm_scratch);
// Fill per-row metadata: seq[i] = i / n, pos[i] = pos0 + i % n.
void fill_row_meta(int *seq, int *pos, int rows, int n, int pos0, cudaStream_t s);
// Identity block table: bt[b][p] = b * pages + p.
void fill_block_table(int *bt, int batch, int pages, cudaStream_t s);

// ---------------------------------------------------------------- megakernel.cu
// One decode step of the engine as a single persistent cooperative kernel
// (batch <= 8, Q8_0 weights, fp16 activations).
struct MkLayer {
    const uint8_t *qkv, *o, *fc, *down;
    const float *attn_norm, *ffn_norm;
    void *kpool, *vpool;
};
struct MkArgs {
    int L, d, H, Hk, D, F, V, B;
    float eps;
    int max_pages, lpad;            // KV block-table width; score row length (>= context, multiple of 64)
    const MkLayer *layers;          // device [L]
    const CUtensorMap *maps;        // device [4 L + 1]: per layer qkv, o, fc (8-row boxes), down; then logits
    const uint8_t *embd;
    int embd_type, vocab_total;
    const float *out_norm, *freqs;
    const int *block_table, *seq;
    int *ids, *pos, *tokens;        // [B]: inputs, positions (advanced by the kernel), outputs
    __half *x, *q, *att, *h;        // activations [B][d], [B][H D], [B][H D], [B][F]
    float *part_val;                // [grid][8] logits winners per CTA
    unsigned long long *part_key;
    int warp_tile_min;              // g_rt.warp_tile_min (see warp_tiles)
    unsigned long long *bar;        // grid barrier counter (monotonic across launches)
    unsigned long long bar_base;    // its value when this launch starts
    int *err;
};
// Grid barriers per launch (arrivals per CTA).
inline int mk_barriers(int L) { return 5 * L + 2; }
// Shared memory of the kernel for `stages` weight units in flight per warp (0 if it does not fit).
size_t mk_smem_bytes(const MkArgs &a, int stages);
// Cooperative launch on every SM; an error (nothing launched) when the device cannot co-schedule it.
cudaError_t mk_launch(const MkArgs &a, int stages, size_t smem, cudaStream_t s);
// A model's map table is being freed: the next launch reloads the constant bank.
void mk_forget_maps(const CUtensorMap *maps);

// ---------------------------------------------------------------- tp.cu
// Tensor parallelism over NCCL (one process per GPU); inactive until wk_tp_init.
bool tp_active();
int tp_rank();
int tp_world();
// in-place fp32 sum over the ranks
void tp_allreduce_f32(float *buf, size_t n, cudaStream_t s);
// bytes of one rank's logits winners for B rows: keys [B] u64, then values [B] f32
size_t tp_winner_chunk(int B);
// all-gather every rank's winners (send: one chunk, recv: world chunks) and
// write the token of the best one per row
void tp_argmax_combine(int *tokens, const void *send, void *recv, int B, int pack, cudaStream_t s);
// x = T(x + T(p)) over n elements
template <typename T> void resid_from_partial(T *x, const float *p, long n, cudaStream_t s);
// Sum the fp32 partials p of all ranks and add them to the residual stream:
// x = T(x + T(sum)).  One fused launch over peer memory when the exchange is
// mapped (decode sizes), else NCCL all-reduce + residual kernel.  Returns this
// library's kernel launches.
template <typename T> int allreduce_resid(T *x, float *p, long n, cudaStream_t s);

// ---------------------------------------------------------------- engine.cu
// Records the message returned by wk_last_error() and returns -1.
int fail(const char *fmt, ...);

// ---------------------------------------------------------------- layers.cu
void layers_init();
void layers_fini();
void prefix_cache_forget(const void *ptr);
void prefix_cache_note_upload(void *dst, const void *src, size_t size);
void prefix_cache_note_write(void *dst, size_t size);
void prefix_cache_embedding(void *out, const int *ids, const void *embd, int batch, int row, int col, int dtype);

}  // namespace wk
