// Native Llama-3 decode engine (wukong_ext.h): paged KV cache, batched greedy
// decode, CUDA-graph replay of the decode step with on-device token feedback.
//
// One decode step for B sequences is 5 launches per layer plus 3:
//   embed (gather + convert) -> per layer { QKV GEMV [RMSNorm | RoPE + KV append],
//   attention, O GEMV [+residual], FC GEMV [RMSNorm | SwiGLU], down GEMV
//   [+residual] } -> logits GEMV [RMSNorm | argmax] -> advance (ids <- tokens,
//   pos += 1).
// The GEMVs and attention are launched with programmatic dependent launch, so
// inside the graph each kernel starts streaming its weights while the previous
// one drains.  The reference computes the same step by re-running the whole
// sequence through cuda.h (llm/llama.go:117-154, llm/model.go:158).
#include <stdarg.h>
#include <stdlib.h>

#include "common.cuh"
#include "wukong_ext.h"
#include "wukong_internal.cuh"

namespace wk {

static char g_err[512] = "";

int fail(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return -1;
}

namespace {

#define WK_TRY(call)                                                                 \
    do {                                                                             \
        cudaError_t e_ = (call);                                                     \
        if (e_ != cudaSuccess) return fail("%s: %s", #call, cudaGetErrorString(e_)); \
    } while (0)

constexpr int kPage = 64;

struct Layer {
    const float *attn_norm = nullptr, *ffn_norm = nullptr;
    const uint8_t *qkv = nullptr, *o = nullptr, *fc = nullptr, *down = nullptr;
};

// ------------------------------------------------------------ small kernels
__global__ void advance_kernel(int *ids, const int *tokens, int *pos, int batch) {
    int b = threadIdx.x + blockIdx.x * blockDim.x;
    if (b < batch) {
        ids[b] = tokens[b];
        pos[b] += 1;
    }
}

// rows[r] of src -> row r of dst (rows of row_u4 16-byte words)
__global__ void gather_rows_by_index_kernel(uint4 *__restrict__ dst, const uint4 *__restrict__ src,
                                            const int *__restrict__ rows, int row_u4) {
    const int r = blockIdx.x;
    const long from = (long)rows[r] * row_u4;
    for (int i = threadIdx.x; i < row_u4; i += blockDim.x) dst[(long)r * row_u4 + i] = src[from + i];
}

__global__ void iota_kernel(int *p, int n, int v0, int step) {
    int i = threadIdx.x + blockIdx.x * blockDim.x;
    if (i < n) p[i] = v0 + i * step;
}

__global__ void fill_i32_kernel(int *p, int n, int v) {
    int i = threadIdx.x + blockIdx.x * blockDim.x;
    if (i < n) p[i] = v;
}

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
// Irwin-Hall(4) of 16-bit uniforms, integer exact (matches the CPU oracle bit for bit)
__device__ __forceinline__ float gen_one(uint64_t seed, uint64_t idx, float k) {
    uint64_t h = mix64(seed + (idx + 1) * 0x9E3779B97F4A7C15ull);
    int32_t s = (int32_t)(h & 0xffff) + (int32_t)((h >> 16) & 0xffff) + (int32_t)((h >> 32) & 0xffff) +
                (int32_t)((h >> 48) & 0xffff);
    return (float)(s - 131070) * k;
}

__global__ void fill_q8_0_kernel(uint8_t *dst, long nblk, uint64_t seed, float k) {
    long b = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblk) return;
    float x[32];
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        x[i] = gen_one(seed, (uint64_t)(b * 32 + i), k);
        amax = fmaxf(amax, fabsf(x[i]));
    }
    const float d = amax / 127.0f;
    // the block is 2-byte aligned: seventeen 16-bit words (scale, then pairs of quants)
    unsigned short *o = reinterpret_cast<unsigned short *>(dst + b * 34);
    o[0] = __half_as_ushort(__float2half_rn(d));
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
        const float q0 = d != 0.f ? fminf(127.f, fmaxf(-127.f, roundf(x[i] / d))) : 0.f;
        const float q1 = d != 0.f ? fminf(127.f, fmaxf(-127.f, roundf(x[i + 1] / d))) : 0.f;
        o[1 + i / 2] = (unsigned short)((uint8_t)(int8_t)q0 | ((unsigned)(uint8_t)(int8_t)q1 << 8));
    }
}

// GGUF Q4_0 quantisation of the same normal samples (the published ggml
// rule): d = (value of largest magnitude) / -8, n = min(15, (int)(x / d + 8.5)).
__global__ void fill_q4_0_kernel(uint8_t *dst, long nblk, uint64_t seed, float k) {
    long b = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblk) return;
    float x[32];
    float amax = 0.f, mx = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        x[i] = gen_one(seed, (uint64_t)(b * 32 + i), k);
        if (fabsf(x[i]) > amax) {
            amax = fabsf(x[i]);
            mx = x[i];
        }
    }
    const float d = mx / -8.0f;
    const float id = d != 0.f ? 1.0f / d : 0.f;
    // the block is 2-byte aligned: nine 16-bit words (scale, then byte pairs of nibbles)
    unsigned short *o = reinterpret_cast<unsigned short *>(dst + b * kQ4Bytes);
    o[0] = __half_as_ushort(__float2half_rn(d));
#pragma unroll
    for (int i = 0; i < 16; i += 2) {
        // separately rounded product and sum (no fused multiply-add), as the host rule
        const int a0 = min(15, (int)__fadd_rn(__fmul_rn(x[i], id), 8.5f));
        const int a1 = min(15, (int)__fadd_rn(__fmul_rn(x[i + 16], id), 8.5f));
        const int b0 = min(15, (int)__fadd_rn(__fmul_rn(x[i + 1], id), 8.5f));
        const int b1 = min(15, (int)__fadd_rn(__fmul_rn(x[i + 17], id), 8.5f));
        o[1 + i / 2] = (unsigned short)((a0 | (a1 << 4)) | ((b0 | (b1 << 4)) << 8));
    }
}

__global__ void fill_f16_kernel(__half *dst, long n, uint64_t seed, float k) {
    long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) dst[i] = __float2half_rn(gen_one(seed, (uint64_t)i, k));
}

__global__ void fill_f32_kernel(float *dst, long n, float v) {
    long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) dst[i] = v;
}

template <typename T> struct IsHalf {
    static constexpr bool value = false;
};
template <> struct IsHalf<__half> {
    static constexpr bool value = true;
};

// token gather converted to the activation type (F32 / F16 / BF16 / Q8_0 tables)
template <typename T>
__global__ void embed_kernel(T *__restrict__ out, const int *__restrict__ ids, const uint8_t *__restrict__ table,
                             int col, int dtype, int vocab, int *err) {
    const int r = blockIdx.x;
    long id = ids[r];
    if (id < 0 || id >= vocab) {
        // an out-of-range id (e.g. -1 from an all-NaN argmax) is reported, never dereferenced
        if (threadIdx.x == 0 && err) atomicCAS(err, 0, 2);
        id = 0;
    }
    if (dtype == (sizeof(T) == 2 ? (IsHalf<T>::value ? kF16 : kBF16) : -1) && (col % 8) == 0) {
        // same 16-bit type: straight 16-byte copies
        const uint4 *src = reinterpret_cast<const uint4 *>(table + id * col * 2);
        uint4 *dst = reinterpret_cast<uint4 *>(out + (long)r * col);
        for (int i = threadIdx.x; i < col / 8; i += blockDim.x) dst[i] = src[i];
        return;
    }
    for (int i = threadIdx.x; i < col; i += blockDim.x) {
        float v;
        if (dtype == kQ8_0) {
            const uint8_t *blk = table + (id * (col / 32) + i / 32) * 34;
            const float s = __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
            v = __half2float(__float2half_rn(s * (float)(int8_t)blk[2 + (i & 31)]));
        } else if (dtype == kQ4_0) {
            const uint8_t *blk = table + (id * (col / 32) + i / 32) * kQ4Bytes;
            const float s = __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
            const int j = i & 31;
            const int nib = j < 16 ? (blk[2 + j] & 15) : (blk[2 + j - 16] >> 4);
            v = __half2float(__float2half_rn(s * (float)(nib - 8)));
        } else if (dtype == kF16) {
            v = __half2float(reinterpret_cast<const __half *>(table)[id * col + i]);
        } else if (dtype == kBF16) {
            v = __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(table)[id * col + i]);
        } else {
            v = reinterpret_cast<const float *>(table)[id * col + i];
        }
        out[(long)r * col + i] = from_float<T>(v);
    }
}

}  // namespace
}  // namespace wk

using namespace wk;

struct wk_model {
    wk_config cfg;
    int act = kF16;
    Layer *layers = nullptr;
    const uint8_t *embd = nullptr, *out_w = nullptr;
    const float *out_norm = nullptr, *freqs = nullptr;
    int freqs_ctx = 0;
    // paged cache: pool[l] = [max_batch * max_pages][Hk][kPage][D]
    int max_batch = 0, max_ctx = 0, max_pages = 0;
    void **kpool = nullptr, **vpool = nullptr;
    int *block_table = nullptr;
    // decode state
    int batch = 0, pos = 0;
    int *d_pos = nullptr, *d_seq = nullptr, *d_ids = nullptr, *d_tokens = nullptr;
    int *d_row_seq = nullptr, *d_row_pos = nullptr;
    // activations
    int rows_cap = 0;
    void *x = nullptr, *q = nullptr, *att = nullptr, *h = nullptr;
    void *xn = nullptr;  // RMSNorm output when a linear layer runs on the tcgen05 GEMM
    // tensor parallelism: this model holds one rank's shard (wk_model_set_tp)
    int tp = 0;
    TpLink link;                                    // peer exchange (link.world > 1) or NCCL (link.world == 1)
    float *p32 = nullptr;                           // [rows_cap, d] fp32 partials of o / down
    void *win_send = nullptr, *win_recv = nullptr;  // logits winners of this rank / of all ranks
    AttnSplitWs attn_ws;                             // split-K decode attention scratch
    // logits argmax partials
    float *part_val = nullptr;
    unsigned long long *part_key = nullptr;
    int *counter = nullptr;
    cudaGraphExec_t graph = nullptr;
    int graph_batch = 0;
    int step_launches = 0;
    // persistent decode kernel (megakernel.cu): -1 not decided, 0 off, 1 on
    int mk_mode = -1;
    MkArgs mk;
    MkLayer *d_mk_layers = nullptr;
    CUtensorMap *d_mk_maps = nullptr;
    unsigned long long *d_mk_bar = nullptr;
    unsigned long long mk_base = 0;
    int mk_stages = 0;
    size_t mk_smem = 0;
    // continuous batching: decode row r serves the sequence in slot row_slot[r]
    // (d_seq on the device); slot_pos holds each slot's length on the host
    int *row_slot = nullptr, *slot_pos = nullptr;
    unsigned char *slot_used = nullptr;
    int *d_meta = nullptr;  // staging of per-row metadata uploads [4 * rows_cap + 4 * max_batch]
    // sampling instead of the fused argmax (wk_model_set_sampling)
    int sampling = 0;
    SampleArgs sample;
    void *logits = nullptr;  // [max_batch, vocab] logits of the last rows
};

namespace {

int ensure_rows(wk_model *m, int rows) {
    if (rows <= m->rows_cap) return 0;
    const wk_config &c = m->cfg;
    const size_t es = act_size(m->act);
    cudaStream_t s = stream();
    for (void **p : {&m->x, &m->q, &m->att, &m->h, &m->xn})
        if (*p) WK_TRY(cudaFreeAsync(*p, s));
    for (int **p : {&m->d_row_seq, &m->d_row_pos})
        if (*p) WK_TRY(cudaFreeAsync(*p, s));
    WK_TRY(cudaMallocAsync(&m->x, es * rows * c.d_model, s));
    WK_TRY(cudaMallocAsync(&m->q, es * rows * c.n_heads * c.head_dim, s));
    WK_TRY(cudaMallocAsync(&m->att, es * rows * c.n_heads * c.head_dim, s));
    WK_TRY(cudaMallocAsync(&m->h, es * rows * c.ffn, s));
    WK_TRY(cudaMallocAsync(&m->xn, es * rows * c.d_model, s));
    if (m->tp) {
        if (m->p32) WK_TRY(cudaFreeAsync(m->p32, s));
        WK_TRY(cudaMallocAsync(&m->p32, sizeof(float) * rows * c.d_model, s));
    }
    WK_TRY(cudaMallocAsync(&m->d_row_seq, sizeof(int) * rows, s));
    WK_TRY(cudaMallocAsync(&m->d_row_pos, sizeof(int) * rows, s));
    m->rows_cap = rows;
    return 0;
}

// Tensor parallelism: sum the o / down partials of all ranks and add them to
// the residual stream.  Returns the number of this library's kernel launches.
int reduce_partials(wk_model *m, int rows, cudaStream_t s) {
    const long n = (long)rows * m->cfg.d_model;
    if (m->act == kF16) return allreduce_resid<__half>((__half *)m->x, m->p32, n, s);
    return allreduce_resid<__nv_bfloat16>((__nv_bfloat16 *)m->x, m->p32, n, s);
}

// Run the layers and the logits head on `rows` activation rows in m->x.
// Row i belongs to sequence seq[i] at position pos[i]; max_len bounds the
// attention length.  Returns the number of kernel launches.

// Prefill of sequences of different lengths (continuous batching): group i
// holds activation rows [row0[i], row0[i] + len[i]) of the sequence in slot
// slot[i], positions 0..len[i]-1; last_rows / last_pos (device) list each
// group's last row and its position.
struct PrefillGroups {
    int count = 0;
    const int *row0 = nullptr, *len = nullptr, *slot = nullptr;  // host
    const int *last_rows = nullptr, *last_pos = nullptr;         // device
};

int run_layers(wk_model *m, int rows, const int *seq, const int *pos, int max_len, int batch, int last_row_stride,
               int *tokens, const PrefillGroups *pg = nullptr) {
    const wk_config &c = m->cfg;
    const size_t es = act_size(m->act);
    const int d = c.d_model, col = c.n_heads * c.head_dim;
    cudaStream_t s = stream();
    PagedKV kv;
    kv.block_table = m->block_table;
    kv.max_pages = m->max_pages;
    kv.page = kPage;
    kv.kv_heads = c.n_kv_heads;
    kv.hd = c.head_dim;
    int launches = 0;
    // L2 prefetch plan: each linear layer streams the weights of the next one
    // (qkv -> o, o -> fc, fc -> down, down -> next qkv); the last down
    // prefetches the head of the logits matrix.  Attention prefetches nothing
    // (its few CTAs would queue the prefetches ahead of their own page loads).
    auto wbytes = [&](long rows, int K, int wt) -> long { return rows * quant_row_bytes(wt, K); };
    // At most g_rt.l2_prefetch_max bytes ahead (12 MB; WUKONG_L2_PREFETCH_MB):
    // a larger prefetch queues ahead of the next kernel's own activation loads
    // in the memory system (measured, 8B: 58 MB ahead of up|gate delayed its
    // prologue by ~5 us; 12 MB: 2.79 -> 2.67 ms/step)
    const long pf_max = g_rt.l2_prefetch_max;
    auto capped = [pf_max](long b) -> long { return b < pf_max ? b : pf_max; };
    const int W = (c.n_heads + 2 * c.n_kv_heads) * c.head_dim;
    // Below kTcMinRows every linear layer here runs on the GEMV, so the launch
    // before each GEMV is a GEMV, an attention kernel (both trigger their
    // dependents after their own wait) or a plain launch: what the launch
    // before that wrote is complete when the GEMV starts, and the GEMV may read
    // its side inputs before its wait
    const int pre = rows < kTcMinRows;
    // tensor-parallel decode rows: the o / down GEMVs exchange their partial
    // tiles with the other ranks and add the residual themselves (ARESID), and
    // the logits GEMV exchanges its winners; more rows (prefill, large
    // batches) run the tcgen05 GEMM, an all-reduce launch and the residual
    const bool fused_ar = m->tp && m->link.world > 1 && rows < kTcMinRows &&
                          (d + 15) / 16 <= kTpMaxTiles;
    const long logit_bytes = wbytes(c.vocab, d, c.out_wtype);
    const long logit_pf = logit_bytes < (48L << 20) ? logit_bytes : (48L << 20);
    for (int l = 0; l < c.n_layers; ++l) {
        const Layer &L = m->layers[l];
        const bool last = l + 1 == c.n_layers;
        kv.k = m->kpool[l];
        kv.v = m->vpool[l];
        {
            GemvArgs a;
            a.w = L.qkv;
            a.wtype = c.wtype;
            a.N = W;
            a.K = d;
            a.x = m->x;
            a.ldx = d;
            a.norm_w = L.attn_norm;
            a.eps = c.eps;
            a.epi = EPI_QKV;
            a.out = m->q;
            a.ldo = col;
            a.nq = c.n_heads * c.head_dim;
            a.nk = c.n_kv_heads * c.head_dim;
            a.hd = c.head_dim;
            a.freqs = m->freqs;
            a.pos = pos;
            a.seq = seq;
            a.kpool = kv.k;
            a.vpool = kv.v;
            a.block_table = kv.block_table;
            a.max_pages = kv.max_pages;
            a.page = kPage;
            a.kv_heads = c.n_kv_heads;
            a.pre = pre;
            a.pf = L.o;
            a.pf_bytes = capped(wbytes(d, col, c.wtype));
            launches += linear(a, rows, m->act, s, m->xn);
        }
        // prefill: batch sequences of last_row_stride positions from 0, flash-style
        int pf = -1;
        if (pg) {
            // each new sequence over its own slot's pages
            pf = 0;
            for (int i = 0; i < pg->count && pf >= 0; ++i) {
                PagedKV kg = kv;
                kg.block_table = kv.block_table + (long)pg->slot[i] * kv.max_pages;
                const size_t o = (size_t)pg->row0[i] * col * es;
                const int r = m->act == kF16
                                  ? attention_prefill_paged<__half>((__half *)((char *)m->att + o), col,
                                                                    (const __half *)((const char *)m->q + o), col, 1,
                                                                    pg->len[i], 0, kg, c.n_heads, s)
                                  : attention_prefill_paged<__nv_bfloat16>(
                                        (__nv_bfloat16 *)((char *)m->att + o), col,
                                        (const __nv_bfloat16 *)((const char *)m->q + o), col, 1, pg->len[i], 0, kg,
                                        c.n_heads, s);
                pf = r < 0 ? -1 : pf + r;
            }
            // shapes the flash kernel does not take: the per-row kernel over all rows (after any
            // launched groups, which it simply recomputes)
            if (pf > 0) launches += pf;
        } else if (rows > batch && rows == batch * last_row_stride) {
            if (m->act == kF16)
                pf = attention_prefill_paged<__half>((__half *)m->att, col, (const __half *)m->q, col, batch,
                                                     last_row_stride, 0, kv, c.n_heads, s);
            else
                pf = attention_prefill_paged<__nv_bfloat16>((__nv_bfloat16 *)m->att, col,
                                                            (const __nv_bfloat16 *)m->q, col, batch, last_row_stride,
                                                            0, kv, c.n_heads, s);
            if (pf > 0) launches += pf;
        }
        if (pf < 0) {
            // decode rows may split the context over several CTAs (split-K attention)
            const AttnSplitWs *ws = rows == batch ? &m->attn_ws : nullptr;
            if (m->act == kF16)
                launches += attention_paged<__half>((__half *)m->att, col, (const __half *)m->q, col, seq, pos, rows,
                                                    max_len, kv, c.n_heads, s, true, nullptr, 0, rows == batch, ws);
            else
                launches += attention_paged<__nv_bfloat16>((__nv_bfloat16 *)m->att, col, (const __nv_bfloat16 *)m->q,
                                                           col, seq, pos, rows, max_len, kv, c.n_heads, s, true,
                                                           nullptr, 0, rows == batch, ws);
        }
        {
            GemvArgs a;
            a.w = L.o;
            a.wtype = c.wtype;
            a.N = d;
            a.K = col;
            a.x = m->att;
            a.ldx = col;
            if (fused_ar) {
                a.epi = EPI_ARESID;
                a.out = m->x;
                a.ldo = d;
                a.res = m->x;
                a.ldr = d;
                a.pre = pre;
                a.tp = m->link;
            } else if (m->tp) {
                a.epi = EPI_PARTIAL;
                a.out = m->p32;
                a.ldo = d;
            } else {
                a.epi = EPI_RESID;
                a.out = m->x;
                a.ldo = d;
                a.res = m->x;
                a.ldr = d;
                a.pre = pre;
            }
            a.pf = L.fc;
            a.pf_bytes = capped(wbytes(2L * c.ffn, d, c.wtype) / 2);
            launches += linear(a, rows, m->act, s, nullptr);
            if (m->tp && !fused_ar) launches += reduce_partials(m, rows, s);
        }
        {
            GemvArgs a;
            a.w = L.fc;
            a.wtype = c.wtype;
            a.N = 2 * c.ffn;
            a.K = d;
            a.x = m->x;
            a.ldx = d;
            a.norm_w = L.ffn_norm;
            a.eps = c.eps;
            a.epi = EPI_SWIGLU;
            a.F = c.ffn;
            a.out = m->h;
            a.ldo = c.ffn;
            a.pf = L.down;
            a.pf_bytes = capped(wbytes(d, c.ffn, c.wtype));
            launches += linear(a, rows, m->act, s, m->xn);
        }
        {
            GemvArgs a;
            a.w = L.down;
            a.wtype = c.wtype;
            a.N = d;
            a.K = c.ffn;
            a.x = m->h;
            a.ldx = c.ffn;
            if (fused_ar) {
                a.epi = EPI_ARESID;
                a.out = m->x;
                a.ldo = d;
                a.res = m->x;
                a.ldr = d;
                a.pre = pre;
                a.tp = m->link;
            } else if (m->tp) {
                a.epi = EPI_PARTIAL;
                a.out = m->p32;
                a.ldo = d;
            } else {
                a.epi = EPI_RESID;
                a.out = m->x;
                a.ldo = d;
                a.res = m->x;
                a.ldr = d;
                a.pre = pre;
            }
            a.pf = last ? (const void *)m->out_w : (const void *)m->layers[l + 1].qkv;
            a.pf_bytes = last ? logit_pf : capped(wbytes(W, d, c.wtype));
            launches += linear(a, rows, m->act, s, nullptr);
            if (m->tp && !fused_ar) launches += reduce_partials(m, rows, s);
        }
    }
    // logits + argmax on the last row of each sequence
    const void *xlast = m->x;
    if (pg) {
        // the groups' last rows, gathered into one [batch, d] block
        gather_rows_by_index_kernel<<<batch, 128, 0, s>>>((uint4 *)m->xn, (const uint4 *)m->x, pg->last_rows,
                                                          (int)(d * es / 16));
        WK_CHECK_LAUNCH();
        ++launches;
        xlast = m->xn;
        last_row_stride = 1;
    }
    for (int b0 = 0; b0 < batch; b0 += 8, ++launches) {
        GemvArgs a;
        a.w = m->out_w;
        a.wtype = c.out_wtype;
        a.N = c.vocab;
        a.K = d;
        a.x = (const char *)xlast + ((size_t)b0 * last_row_stride + (last_row_stride - 1)) * d * es;
        a.ldx = (long)last_row_stride * d;
        a.M = batch - b0 < 8 ? batch - b0 : 8;
        a.norm_w = m->out_norm;
        a.eps = c.eps;
        a.epi = EPI_LOGITS;
        a.part_val = m->part_val;
        a.part_key = m->part_key;
        a.counter = m->counter;
        a.pack = 16 / (int)es;
        if (m->tp) {
            // vocabulary shard: keys in whole-vocabulary columns
            a.col_off = (long)tp_rank() * c.vocab;
            a.n_total = c.vocab * tp_world();
            if (m->link.world > 1) {
                // the winners are exchanged by the GEMV's last CTA
                a.tp = m->link;
                a.tokens = tokens + b0;
            } else {
                // winners exchanged below
                a.best_key = (unsigned long long *)m->win_send + b0;
                a.best_val = (float *)((char *)m->win_send + 8L * batch) + b0;
            }
        } else {
            a.tokens = tokens + b0;
            if (m->sampling) {
                a.out = (char *)m->logits + (size_t)b0 * c.vocab * es;
                a.ldo = c.vocab;
            }
        }
        gemv(a, m->act, s);
    }
    if (m->sampling && !m->tp) {
        // the draw replaces the argmax; RNG step = the position of each sequence's last row
        SampleArgs sp = m->sample;
        sp.pos = pg ? pg->last_pos : pos;
        sp.pos_stride = pg ? 1 : last_row_stride;
        sp.pos_off = pg ? 0 : last_row_stride - 1;
        sample_rows(tokens, m->logits, c.vocab, batch, c.vocab, m->act, sp, s);
        ++launches;
    }
    if (m->tp && m->link.world == 1) {
        tp_argmax_combine(tokens, m->win_send, m->win_recv, batch, 16 / (int)es, s);
        ++launches;
    }
    return launches;
}

// Decide once per model whether decode steps run as the persistent kernel
// (opt-in: WUKONG_MEGAKERNEL=1), and build its per-layer tables and weight
// tensor maps.  Not for tensor-parallel shards or shapes it does not take
// (Q8_0 linear and output weights, K multiples of 256, head_dim 64 / 128, at
// most 8 query heads per KV head, a context whose scores fit in shared memory).
void mk_setup(wk_model *m) {
    m->mk_mode = 0;
    const char *env = getenv("WUKONG_MEGAKERNEL");
    if (!env || env[0] != '1') return;
    const wk_config &c = m->cfg;
    const int D = c.head_dim, W = (c.n_heads + 2 * c.n_kv_heads) * D;
    if (m->tp || m->act != kF16 || c.wtype != kQ8_0 || c.out_wtype != kQ8_0) return;
    if (c.d_model % 256 || (c.n_heads * D) % 256 || c.ffn % 256 || (D != 64 && D != 128)) return;
    if (c.n_heads % c.n_kv_heads || c.n_heads / c.n_kv_heads > 8 || !m->kpool) return;
    if (c.embd_wtype != kF32 && c.embd_wtype != kF16 && c.embd_wtype != kBF16 && c.embd_wtype != kQ8_0) return;
    MkArgs a = {};
    a.L = c.n_layers;
    a.d = c.d_model;
    a.H = c.n_heads;
    a.Hk = c.n_kv_heads;
    a.D = D;
    a.F = c.ffn;
    a.V = c.vocab;
    a.B = 8;  // shared memory is sized for the largest batch
    a.eps = c.eps;
    a.max_pages = m->max_pages;
    a.lpad = (m->max_ctx + kPage - 1) / kPage * kPage;
    int S = 0;
    size_t smem = 0;
    for (int st = 5; st >= 2 && !smem; --st) {
        smem = mk_smem_bytes(a, st);
        S = st;
    }
    if (!smem) return;
    // tensor maps: qkv, o, fc (8-row boxes: up and gate halves), down per layer, then logits
    const int L = c.n_layers;
    CUtensorMap *maps = (CUtensorMap *)aligned_alloc(64, sizeof(CUtensorMap) * (4 * L + 1));
    MkLayer *layers = (MkLayer *)calloc(L, sizeof(MkLayer));
    bool ok = maps && layers;
    auto enc = [&](CUtensorMap *mp, const void *w, long rows, int K, int box_rows) {
        const long rb = (long)(K / 32) * 34;
        ok = ok && ((uintptr_t)w % 16) == 0 &&
             encode_map_2d(mp, w, CU_TENSOR_MAP_DATA_TYPE_UINT16, (uint64_t)rb / 2, (uint64_t)rows, (uint64_t)rb, 136,
                           (uint32_t)box_rows, CU_TENSOR_MAP_SWIZZLE_NONE);
    };
    for (int l = 0; ok && l < L; ++l) {
        const Layer &Ly = m->layers[l];
        enc(maps + 4 * l + 0, Ly.qkv, W, c.d_model, 16);
        enc(maps + 4 * l + 1, Ly.o, c.d_model, c.n_heads * D, 16);
        enc(maps + 4 * l + 2, Ly.fc, 2L * c.ffn, c.d_model, 8);
        enc(maps + 4 * l + 3, Ly.down, c.d_model, c.ffn, 16);
        layers[l] = MkLayer{Ly.qkv, Ly.o, Ly.fc, Ly.down, Ly.attn_norm, Ly.ffn_norm, m->kpool[l], m->vpool[l]};
    }
    if (ok) enc(maps + 4 * L, m->out_w, c.vocab, c.d_model, 16);
    if (ok) ok = cudaMalloc(&m->d_mk_maps, sizeof(CUtensorMap) * (4 * L + 1)) == cudaSuccess &&
                 cudaMalloc(&m->d_mk_layers, sizeof(MkLayer) * L) == cudaSuccess &&
                 cudaMalloc(&m->d_mk_bar, sizeof(unsigned long long)) == cudaSuccess &&
                 cudaMemcpy(m->d_mk_maps, maps, sizeof(CUtensorMap) * (4 * L + 1), cudaMemcpyHostToDevice) ==
                     cudaSuccess &&
                 cudaMemcpy(m->d_mk_layers, layers, sizeof(MkLayer) * L, cudaMemcpyHostToDevice) == cudaSuccess &&
                 cudaMemset(m->d_mk_bar, 0, sizeof(unsigned long long)) == cudaSuccess;
    free(maps);
    free(layers);
    if (!ok) {
        cudaGetLastError();
        return;
    }
    a.layers = m->d_mk_layers;
    a.maps = m->d_mk_maps;
    a.embd = m->embd;
    a.embd_type = c.embd_wtype;
    a.vocab_total = c.vocab;
    a.out_norm = m->out_norm;
    a.freqs = m->freqs;
    a.block_table = m->block_table;
    a.seq = m->d_seq;
    a.part_val = m->part_val;
    a.part_key = m->part_key;
    a.bar = m->d_mk_bar;
    a.err = g_rt.d_error;
    a.warp_tile_min = g_rt.warp_tile_min;
    m->mk = a;
    m->mk_stages = S;
    m->mk_smem = smem;
    m->mk_base = 0;
    m->mk_mode = 1;
}

void launch_embed(wk_model *m, const int *ids, int rows) {
    const wk_config &c = m->cfg;
    // the token table is whole on every rank; a shard's vocab counts only its logits rows
    const int vocab = m->tp ? c.vocab * tp_world() : c.vocab;
    if (m->act == kF16)
        embed_kernel<__half><<<rows, 256, 0, stream()>>>((__half *)m->x, ids, m->embd, c.d_model, c.embd_wtype,
                                                         vocab, g_rt.d_error);
    else
        embed_kernel<__nv_bfloat16><<<rows, 256, 0, stream()>>>((__nv_bfloat16 *)m->x, ids, m->embd, c.d_model,
                                                                c.embd_wtype, vocab, g_rt.d_error);
    WK_CHECK_LAUNCH();
}

}  // namespace

extern "C" {

const char *wk_last_error(void) { return g_err; }

void *wk_stream(void) { return (void *)stream(); }

wk_model *wk_model_create(const wk_config *cfg) {
    if (g_rt.device < 0) {
        fail("cuda_init() has not been called");
        return nullptr;
    }
    set_device_current();
    const wk_config &c = *cfg;
    // n_heads * head_dim is d_model, or d_model / world for a tensor-parallel shard
    if (c.n_kv_heads <= 0 || c.n_heads <= 0 || c.n_heads % c.n_kv_heads || c.head_dim % 2 ||
        c.d_model % (c.n_heads * c.head_dim)) {
        fail("inconsistent attention geometry");
        return nullptr;
    }
    const int act = act_of(c.wtype);
    if (act == kF32 || !gemv_supported(c.wtype, act, c.d_model) || !gemv_supported(c.wtype, act, c.ffn) ||
        !gemv_supported(c.out_wtype, act, c.d_model)) {
        fail("the engine needs F16 / BF16 / Q8_0 weights with 16/32-aligned widths");
        return nullptr;
    }
    wk_model *m = new wk_model();  // value-initialised: default member initialisers apply
    m->cfg = c;
    m->act = act;
    m->layers = (Layer *)calloc(c.n_layers, sizeof(Layer));
    cudaStream_t s = stream();
    if (cudaMallocAsync(&m->part_val, sizeof(float) * kMaxLogitCtas * 8, s) != cudaSuccess ||
        cudaMallocAsync(&m->part_key, sizeof(unsigned long long) * kMaxLogitCtas * 8, s) != cudaSuccess ||
        cudaMallocAsync(&m->counter, sizeof(int), s) != cudaSuccess ||
        cudaMemsetAsync(m->counter, 0, sizeof(int), s) != cudaSuccess) {
        fail("allocation failed");
        free(m->layers);
        delete m;
        return nullptr;
    }
    return m;
}

void wk_model_destroy(wk_model *m) {
    if (!m) return;
    set_device_current();
    cudaStream_t s = stream();
    cudaStreamSynchronize(s);
    if (m->graph) cudaGraphExecDestroy(m->graph);
    if (m->d_mk_maps) mk_forget_maps(m->d_mk_maps);
    for (int l = 0; m->kpool && l < m->cfg.n_layers; ++l) {
        cudaFree(m->kpool[l]);
        cudaFree(m->vpool[l]);
    }
    free(m->kpool);
    free(m->vpool);
    void *bufs[] = {m->block_table, m->d_pos, m->d_seq, m->d_ids, m->d_tokens, m->d_row_seq, m->d_row_pos,
                    m->x, m->q, m->att, m->h, m->xn, m->part_val, m->part_key, m->counter,
                    m->p32, m->win_send, m->win_recv, m->d_mk_layers, m->d_mk_maps, m->d_mk_bar,
                    m->attn_ws.scores, m->attn_ws.mpart, m->attn_ws.opart, m->attn_ws.counter,
                    m->attn_ws.minv, m->logits};
    for (void *p : bufs)
        if (p) cudaFree(p);
    if (m->d_meta) cudaFree(m->d_meta);
    free(m->row_slot);
    free(m->slot_pos);
    free(m->slot_used);
    free(m->layers);
    delete m;
}

int wk_model_set_layer(wk_model *m, int l, const void *attn_norm, const void *qkv, const void *o,
                       const void *ffn_norm, const void *fc, const void *down) {
    if (!m || l < 0 || l >= m->cfg.n_layers) return fail("bad layer index %d", l);
    Layer &L = m->layers[l];
    L.attn_norm = (const float *)attn_norm;
    L.qkv = (const uint8_t *)qkv;
    L.o = (const uint8_t *)o;
    L.ffn_norm = (const float *)ffn_norm;
    L.fc = (const uint8_t *)fc;
    L.down = (const uint8_t *)down;
    return 0;
}

int wk_model_set_head(wk_model *m, const void *token_embd, const void *output_norm, const void *output,
                      const void *freqs, int freqs_ctx) {
    if (!m) return fail("null model");
    m->embd = (const uint8_t *)token_embd;
    m->out_norm = (const float *)output_norm;
    m->out_w = (const uint8_t *)output;
    m->freqs = (const float *)freqs;
    m->freqs_ctx = freqs_ctx;
    return 0;
}

int wk_model_alloc_cache(wk_model *m, int max_batch, int max_ctx) {
    if (!m || max_batch <= 0 || max_ctx <= 0) return fail("bad cache size");
    set_device_current();
    const wk_config &c = m->cfg;
    cudaStream_t s = stream();
    m->max_batch = max_batch;
    m->max_ctx = max_ctx;
    m->max_pages = (max_ctx + kPage - 1) / kPage;
    const size_t page_bytes = (size_t)c.n_kv_heads * kPage * c.head_dim * act_size(m->act);
    m->kpool = (void **)calloc(c.n_layers, sizeof(void *));
    m->vpool = (void **)calloc(c.n_layers, sizeof(void *));
    for (int l = 0; l < c.n_layers; ++l) {
        WK_TRY(cudaMalloc(&m->kpool[l], page_bytes * max_batch * m->max_pages));
        WK_TRY(cudaMalloc(&m->vpool[l], page_bytes * max_batch * m->max_pages));
    }
    WK_TRY(cudaMallocAsync(&m->block_table, sizeof(int) * max_batch * m->max_pages, s));
    fill_block_table(m->block_table, max_batch, m->max_pages, s);
    for (int **p : {&m->d_pos, &m->d_seq, &m->d_ids, &m->d_tokens}) WK_TRY(cudaMallocAsync(p, sizeof(int) * max_batch, s));
    iota_kernel<<<(max_batch + 127) / 128, 128, 0, s>>>(m->d_seq, max_batch, 0, 1);
    m->row_slot = (int *)calloc(max_batch, sizeof(int));
    m->slot_pos = (int *)calloc(max_batch, sizeof(int));
    m->slot_used = (unsigned char *)calloc(max_batch, 1);
    WK_TRY(cudaMallocAsync(&m->d_meta, sizeof(int) * 4 * max_batch, s));
    WK_TRY(cudaGetLastError());
    {
        // split-K decode attention: up to 64 splits of the context per (sequence, kv head)
        AttnSplitWs &w = m->attn_ws;
        w.max_rows = max_batch;
        w.max_kv_heads = c.n_kv_heads;
        w.max_splits = 64;
        w.lpad = m->max_pages * kPage;
        const size_t rh = (size_t)max_batch * c.n_kv_heads;
        WK_TRY(cudaMallocAsync(&w.scores, rh * 8 * w.lpad * act_size(m->act), s));
        WK_TRY(cudaMallocAsync((void **)&w.mpart, rh * w.max_splits * 16 * sizeof(float), s));
        WK_TRY(cudaMallocAsync((void **)&w.opart, rh * w.max_splits * 8 * c.head_dim * sizeof(float), s));
        WK_TRY(cudaMallocAsync((void **)&w.counter, 2 * rh * sizeof(int), s));
        WK_TRY(cudaMemsetAsync(w.counter, 0, 2 * rh * sizeof(int), s));
        w.counter_a = w.counter + rh;
        WK_TRY(cudaMallocAsync((void **)&w.minv, rh * 16 * sizeof(float), s));
    }
    if (m->tp) {
        WK_TRY(cudaMallocAsync(&m->win_send, tp_winner_chunk(max_batch), s));
        WK_TRY(cudaMallocAsync(&m->win_recv, tp_winner_chunk(max_batch) * tp_world(), s));
    }
    return 0;
}

int wk_model_set_sampling(wk_model *m, float temperature, int top_k, float top_p, unsigned long long seed) {
    if (!m) return fail("null model");
    if (m->tp && temperature > 0.f) return fail("sampling is not available with tensor parallelism");
    if (!m->kpool) return fail("wk_model_set_sampling must come after wk_model_alloc_cache");
    set_device_current();
    if (temperature > 0.f && !m->logits)
        WK_TRY(cudaMallocAsync(&m->logits, (size_t)m->max_batch * m->cfg.vocab * act_size(m->act), stream()));
    m->sampling = temperature > 0.f ? 1 : 0;
    m->sample = SampleArgs();
    m->sample.temperature = temperature > 0.f ? temperature : 1.f;
    m->sample.top_k = top_k;
    m->sample.top_p = top_p;
    m->sample.seed = seed;
    // the decode graph holds the previous choice
    if (m->graph) {
        WK_TRY(cudaStreamSynchronize(stream()));
        cudaGraphExecDestroy(m->graph);
        m->graph = nullptr;
    }
    return 0;
}

int wk_model_set_tp(wk_model *m, int enable) {
    if (!m) return fail("null model");
    if (m->kpool) return fail("wk_model_set_tp must come before wk_model_alloc_cache");
    if (enable && !tp_active()) return fail("wk_model_set_tp: wk_tp_init has not set up more than one rank");
    m->tp = enable ? 1 : 0;
    m->link = TpLink();
    if (m->tp) tp_link(&m->link);
    return 0;
}

// A bounded device wait that gave up (a lost peer, a copy that never landed)
// left the decode state incomplete: refuse further launches until the host
// has handled it (wk_device_error).  Tensor-parallel ranks are then out of
// step; recovery is wk_tp_fini and a new communicator.
static int device_error_pending() {
    const int e = g_rt.h_error ? *(volatile int *)g_rt.h_error : 0;
    return e ? fail("a device-side bounded wait gave up earlier (code %d); see wk_device_error", e) : 0;
}

int wk_model_prefill(wk_model *m, const int *ids, int batch, int n, int *tokens_out) {
    if (!m || !m->kpool) return fail("cache not allocated");
    if (device_error_pending()) return -1;
    if (batch <= 0 || batch > m->max_batch || n <= 0 || n > m->max_ctx || n > m->freqs_ctx)
        return fail("prefill batch %d x %d exceeds the cache (%d x %d)", batch, n, m->max_batch, m->max_ctx);
    set_device_current();
    const int rows = batch * n;
    if (ensure_rows(m, rows < 8 * batch ? 8 * batch : rows)) return -1;
    cudaStream_t s = stream();
    fill_row_meta(m->d_row_seq, m->d_row_pos, rows, n, 0, s);
    launch_embed(m, ids, rows);
    run_layers(m, rows, m->d_row_seq, m->d_row_pos, n, batch, n, m->d_tokens);
    // arm decode: next inputs are the predicted tokens at position n
    WK_TRY(cudaMemcpyAsync(m->d_ids, m->d_tokens, sizeof(int) * batch, cudaMemcpyDeviceToDevice, s));
    fill_i32_kernel<<<(batch + 127) / 128, 128, 0, s>>>(m->d_pos, batch, n);
    WK_TRY(cudaGetLastError());
    if (tokens_out) WK_TRY(cudaMemcpyAsync(tokens_out, m->d_tokens, sizeof(int) * batch, cudaMemcpyDeviceToDevice, s));
    // the batch is the sequences of slots 0..batch-1, in order
    iota_kernel<<<(batch + 127) / 128, 128, 0, s>>>(m->d_seq, batch, 0, 1);
    WK_TRY(cudaGetLastError());
    memset(m->slot_used, 0, m->max_batch);
    for (int b = 0; b < batch; ++b) {
        m->row_slot[b] = b;
        m->slot_pos[b] = n;
        m->slot_used[b] = 1;
    }
    if (m->graph && m->graph_batch != batch) {
        cudaGraphExecDestroy(m->graph);
        m->graph = nullptr;
    }
    m->batch = batch;
    m->pos = n;
    return 0;
}

// the longest active sequence (the context bound of the next step)
static int longest(const wk_model *m) {
    int p = 0;
    for (int r = 0; r < m->batch; ++r) p = m->slot_pos[m->row_slot[r]] > p ? m->slot_pos[m->row_slot[r]] : p;
    return p;
}

int wk_model_add_seqs(wk_model *m, const int *ids, const int *lens, int count, int *slots_out) {
    if (!m || !m->kpool) return fail("cache not allocated");
    if (device_error_pending()) return -1;
    if (m->tp) return fail("wk_model_add_seqs: not with tensor parallelism");
    if (count <= 0 || !ids || !lens || m->batch + count > m->max_batch)
        return fail("wk_model_add_seqs: %d sequences do not fit beside %d of %d", count, m->batch, m->max_batch);
    int rows = 0, longest_new = 0;
    for (int i = 0; i < count; ++i) {
        if (lens[i] <= 0 || lens[i] > m->max_ctx || lens[i] > m->freqs_ctx)
            return fail("wk_model_add_seqs: length %d outside [1, %d]", lens[i], m->max_ctx);
        rows += lens[i];
        longest_new = lens[i] > longest_new ? lens[i] : longest_new;
    }
    set_device_current();
    cudaStream_t s = stream();
    if (ensure_rows(m, rows < 8 * m->max_batch ? 8 * m->max_batch : rows)) return -1;
    // free slots, lowest first
    int *slot = (int *)malloc(sizeof(int) * count * 3), *row0 = slot + count;
    int *meta = (int *)malloc(sizeof(int) * (2 * rows + 2 * count));
    int *rseq = meta, *rpos = meta + rows, *lrow = meta + 2 * rows, *lpos = lrow + count;
    for (int i = 0, sl = 0; i < count; ++i) {
        while (m->slot_used[sl]) ++sl;
        slot[i] = sl++;
    }
    for (int i = 0, r = 0; i < count; ++i) {
        row0[i] = r;
        for (int j = 0; j < lens[i]; ++j, ++r) {
            rseq[r] = slot[i];
            rpos[r] = j;
        }
        lrow[i] = r - 1;
        lpos[i] = lens[i] - 1;
    }
    // per-row slot and position, then each new sequence's last row and its position
    cudaError_t e = cudaMemcpyAsync(m->d_row_seq, rseq, sizeof(int) * rows, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(m->d_row_pos, rpos, sizeof(int) * rows, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(m->d_meta, lrow, sizeof(int) * 2 * count, cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) {
        free(slot);
        free(meta);
        return fail("wk_model_add_seqs: %s", cudaGetErrorString(e));
    }
    PrefillGroups pg;
    pg.count = count;
    pg.row0 = row0;
    pg.len = lens;
    pg.slot = slot;
    pg.last_rows = m->d_meta;
    pg.last_pos = m->d_meta + count;
    const int B0 = m->batch;
    launch_embed(m, ids, rows);
    run_layers(m, rows, m->d_row_seq, m->d_row_pos, longest_new, count, 1, m->d_tokens + B0, &pg);
    // the new rows join the decode batch: next input = the generated token at position len
    for (int i = 0; i < count; ++i) {
        m->row_slot[B0 + i] = slot[i];
        m->slot_pos[slot[i]] = lens[i];
        m->slot_used[slot[i]] = 1;
        if (slots_out) slots_out[i] = slot[i];
    }
    int *hostv = (int *)malloc(sizeof(int) * 2 * count);
    for (int i = 0; i < count; ++i) {
        hostv[i] = slot[i];
        hostv[count + i] = lens[i];
    }
    e = cudaMemcpyAsync(m->d_seq + B0, hostv, sizeof(int) * count, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(m->d_pos + B0, hostv + count, sizeof(int) * count, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(m->d_ids + B0, m->d_tokens + B0, sizeof(int) * count, cudaMemcpyDeviceToDevice, s);
    free(hostv);
    free(slot);
    free(meta);
    if (e != cudaSuccess) return fail("wk_model_add_seqs: %s", cudaGetErrorString(e));
    m->batch = B0 + count;
    m->pos = longest(m);
    if (m->graph && m->graph_batch != m->batch) {
        cudaGraphExecDestroy(m->graph);
        m->graph = nullptr;
    }
    return 0;
}

int wk_model_remove_seq(wk_model *m, int slot) {
    if (!m || !m->kpool) return fail("cache not allocated");
    if (slot < 0 || slot >= m->max_batch || !m->slot_used[slot]) return fail("wk_model_remove_seq: slot %d is not in use", slot);
    set_device_current();
    cudaStream_t s = stream();
    int r = 0;
    while (m->row_slot[r] != slot) ++r;
    const int L = m->batch - 1;
    if (r != L) {
        // the last row takes the freed row's place
        m->row_slot[r] = m->row_slot[L];
        for (int *p : {m->d_seq, m->d_pos, m->d_ids, m->d_tokens})
            WK_TRY(cudaMemcpyAsync(p + r, p + L, sizeof(int), cudaMemcpyDeviceToDevice, s));
    }
    m->slot_used[slot] = 0;
    m->batch = L;
    m->pos = longest(m);
    if (m->graph) {
        WK_TRY(cudaStreamSynchronize(s));
        cudaGraphExecDestroy(m->graph);
        m->graph = nullptr;
    }
    return 0;
}

int wk_model_rows(const wk_model *m, int *slots) {
    if (!m) return 0;
    if (slots)
        for (int r = 0; r < m->batch; ++r) slots[r] = m->row_slot[r];
    return m->batch;
}

int wk_model_decode_step(wk_model *m) {
    if (!m || m->batch <= 0) return fail("no armed batch (call wk_model_prefill first)");
    if (m->pos + 1 > m->max_ctx || m->pos + 1 > m->freqs_ctx) return fail("context full (%d)", m->pos);
    if (device_error_pending()) return -1;
    set_device_current();
    cudaStream_t s = stream();
    const int B = m->batch;
    for (int r = 0; r < B; ++r) ++m->slot_pos[m->row_slot[r]];
    if (m->graph && m->graph_batch != B) {
        WK_TRY(cudaStreamSynchronize(s));
        cudaGraphExecDestroy(m->graph);
        m->graph = nullptr;
    }
    if (m->mk_mode < 0) mk_setup(m);
    if (m->mk_mode == 1 && B <= 8 && !m->sampling) {
        if (ensure_rows(m, 8 * B)) return -1;
        MkArgs a = m->mk;
        a.B = B;
        a.bar_base = m->mk_base;
        a.ids = m->d_ids;
        a.pos = m->d_pos;
        a.tokens = m->d_tokens;
        a.x = (__half *)m->x;
        a.q = (__half *)m->q;
        a.att = (__half *)m->att;
        a.h = (__half *)m->h;
        const cudaError_t e = mk_launch(a, m->mk_stages, m->mk_smem, s);
        if (e == cudaSuccess) {
            m->mk_base += (unsigned long long)mk_barriers(m->cfg.n_layers) * g_rt.num_sms;
            m->step_launches = 1;
            m->pos = longest(m);
            return 0;
        }
        // the device cannot co-schedule it: use the graph path from now on
        cudaGetLastError();
        fprintf(stderr, "wukong: persistent decode kernel not launched (%s); using the per-op graph\n",
                cudaGetErrorString(e));
        m->mk_mode = 0;
    }
    if (!m->graph) {
        if (ensure_rows(m, 8 * B)) return -1;
        WK_TRY(cudaStreamSynchronize(s));
        cudaGraph_t g;
        WK_TRY(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
        launch_embed(m, m->d_ids, B);
        int n = 1 + run_layers(m, B, m->d_seq, m->d_pos, m->max_ctx, B, 1, m->d_tokens);
        advance_kernel<<<(B + 127) / 128, 128, 0, s>>>(m->d_ids, m->d_tokens, m->d_pos, B);
        n += 1;
        cudaError_t e = cudaGetLastError();
        cudaError_t e2 = cudaStreamEndCapture(s, &g);
        if (e != cudaSuccess || e2 != cudaSuccess)
            return fail("graph capture failed: %s / %s", cudaGetErrorString(e), cudaGetErrorString(e2));
        WK_TRY(cudaGraphInstantiate(&m->graph, g, 0));
        cudaGraphDestroy(g);
        m->graph_batch = B;
        m->step_launches = n;
    }
    WK_TRY(cudaGraphLaunch(m->graph, s));
    m->pos = longest(m);
    return 0;
}

const int *wk_model_tokens(const wk_model *m) { return m ? m->d_tokens : nullptr; }
const void *wk_model_logits(const wk_model *m) { return m && m->sampling ? m->logits : nullptr; }
int *wk_model_next_ids(wk_model *m) { return m ? m->d_ids : nullptr; }
int wk_model_step_launches(const wk_model *m) { return m ? m->step_launches : 0; }
int wk_model_position(const wk_model *m) { return m ? m->pos : 0; }

int wk_model_truncate(wk_model *m, int n) {
    if (!m || m->batch <= 0) return fail("no armed batch (call wk_model_prefill first)");
    int shortest = m->pos;
    for (int r = 0; r < m->batch; ++r)
        shortest = m->slot_pos[m->row_slot[r]] < shortest ? m->slot_pos[m->row_slot[r]] : shortest;
    if (n < 1 || n > shortest) return fail("truncate to %d outside [1, %d]", n, shortest);
    set_device_current();
    cudaStream_t s = stream();
    fill_i32_kernel<<<(m->batch + 127) / 128, 128, 0, s>>>(m->d_pos, m->batch, n);
    WK_TRY(cudaGetLastError());
    for (int r = 0; r < m->batch; ++r) m->slot_pos[m->row_slot[r]] = n;
    m->pos = n;
    return 0;
}

// The engine's decode attention over a paged K/V cache, callable on its own.
int wk_attention_decode(void *out, const void *q, const void *kpool, const void *vpool, const int *block_table,
                        int max_pages, const int *seq, const int *pos, int rows, int max_len, int n_heads,
                        int kv_heads, int head_dim, int dtype) {
    if (g_rt.device < 0) return fail("wk_attention_decode: cuda_init() has not been called");
    if (!out || !q || !kpool || !vpool || !block_table || !seq || !pos || rows < 1 || max_len < 1 || kv_heads < 1 ||
        n_heads % kv_heads || max_pages * kPage < max_len)
        return fail("wk_attention_decode: bad arguments");
    if (dtype != kF16 && dtype != kBF16) return fail("wk_attention_decode: dtype %d", dtype);
    set_device_current();
    PagedKV c;
    c.k = const_cast<void *>(kpool);
    c.v = const_cast<void *>(vpool);
    c.block_table = block_table;
    c.max_pages = max_pages;
    c.page = kPage;
    c.kv_heads = kv_heads;
    c.hd = head_dim;
    const long col = (long)n_heads * head_dim;
    if (dtype == kF16)
        attention_paged<__half>((__half *)out, col, (const __half *)q, col, seq, pos, rows, max_len, c, n_heads,
                                stream(), true, nullptr, 0, true, nullptr);
    else
        attention_paged<__nv_bfloat16>((__nv_bfloat16 *)out, col, (const __nv_bfloat16 *)q, col, seq, pos, rows,
                                       max_len, c, n_heads, stream(), true, nullptr, 0, true, nullptr);
    return 0;
}

int wk_fill_random_q8_0(void *dst, long rows, int cols, uint64_t seed, float stdv) {
    if (cols % 32) return fail("cols must be a multiple of 32");
    ensure_init();
    const long nblk = rows * (cols / 32);
    const float k = stdv / 37837.227f;
    fill_q8_0_kernel<<<(unsigned)((nblk + 255) / 256), 256, 0, stream()>>>((uint8_t *)dst, nblk, seed, k);
    WK_TRY(cudaGetLastError());
    return 0;
}

int wk_fill_random_q4_0(void *dst, long rows, int cols, uint64_t seed, float stdv) {
    if (cols % 32) return fail("cols must be a multiple of 32");
    ensure_init();
    const long nblk = rows * (cols / 32);
    fill_q4_0_kernel<<<(unsigned)((nblk + 255) / 256), 256, 0, stream()>>>((uint8_t *)dst, nblk, seed,
                                                                          stdv / 37837.227f);
    WK_TRY(cudaGetLastError());
    return 0;
}

int wk_fill_random_f16(void *dst, long n, uint64_t seed, float stdv) {
    ensure_init();
    const float k = stdv / 37837.227f;
    fill_f16_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream()>>>((__half *)dst, n, seed, k);
    WK_TRY(cudaGetLastError());
    return 0;
}

int wk_fill_const_f32(void *dst, long n, float value) {
    ensure_init();
    fill_f32_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream()>>>((float *)dst, n, value);
    WK_TRY(cudaGetLastError());
    return 0;
}

int wk_gemv(void *out, const void *x, const void *w, int M, int K, int N, int wtype) {
    ensure_init();
    const int act = act_of(wtype);
    if (M < 1 || M > 8 || !gemv_supported(wtype, act, K)) return fail("wk_gemv: unsupported shape/dtype");
    GemvArgs a;
    a.w = (const uint8_t *)w;
    a.wtype = wtype;
    a.N = N;
    a.K = K;
    a.x = x;
    a.ldx = K;
    a.M = M;
    a.epi = EPI_STORE;
    a.out = out;
    a.ldo = N;
    gemv(a, act, stream());
    return 0;
}

}  // extern "C"
