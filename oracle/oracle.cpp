/*
 * CPU oracle for the wukong hot path -- TEST INFRASTRUCTURE ONLY (see oracle.h).
 *
 * Each function restates one op of the reference's cuda.cu (liuy/wukong) on the
 * CPU, citing the file:line it follows.  The restatement keeps the reference's
 * storage-rounding points (every T-typed buffer write rounds to T) and its fp32
 * accumulation; it does not reproduce cuBLAS's summation order, which is not
 * published.  Built with -ffp-contract=off so that every float operation is a
 * separately rounded IEEE operation.
 */
#include "oracle.h"

#include <math.h>
#include <omp.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <vector>

namespace {

inline float f16_round(float x) { return (float)(_Float16)x; }

inline float bf16_round(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    if ((u & 0x7f800000u) == 0x7f800000u) {
        if (u & 0x007fffffu) u |= 0x00400000u;  // quiet NaN
        u &= 0xffff0000u;
    } else {
        u += 0x7fffu + ((u >> 16) & 1u);  // round to nearest even
        u &= 0xffff0000u;
    }
    memcpy(&x, &u, 4);
    return x;
}

/* cuBLASLt runs F32 GEMMs with CUBLAS_COMPUTE_32F_FAST_TF32 (cuda.cu:1046-1048);
 * the reference's Go end-to-end vectors (llm/array_test.go:827-836) carry TF32
 * inputs rounded to nearest, its gtest vectors exact fp32.  Off by default. */
int g_f32_tf32 = 0;

inline float tf32_rn(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    if ((u & 0x7f800000u) != 0x7f800000u) u = (u + 0xfffu + ((u >> 13) & 1u)) & 0xffffe000u;
    memcpy(&x, &u, 4);
    return x;
}

inline float rnd(int act, float x) {
    if (act == ORC_F16) return f16_round(x);
    if (act == ORC_BF16) return bf16_round(x);
    return x;
}

inline float h2f(uint16_t h) {
    _Float16 v;
    memcpy(&v, &h, 2);
    return (float)v;
}

inline float b2f(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* Decode one weight row into float.  Q8_0 follows cuda_matmul's dequantise-to-half
 * path (cuda.cu:1104-1108): w = (half)(float(scale) * q). */
void decode_row(const void *w, int wtype, long row, int K, float *dst, int q8_round_half) {
    switch (wtype) {
    case ORC_F32:
        memcpy(dst, (const float *)w + row * (long)K, sizeof(float) * K);
        break;
    case ORC_F16: {
        const uint16_t *p = (const uint16_t *)w + row * (long)K;
        for (int k = 0; k < K; ++k) dst[k] = h2f(p[k]);
        break;
    }
    case ORC_BF16: {
        const uint16_t *p = (const uint16_t *)w + row * (long)K;
        for (int k = 0; k < K; ++k) dst[k] = b2f(p[k]);
        break;
    }
    case ORC_Q8_0: {
        const uint8_t *p = (const uint8_t *)w + row * (long)(K / 32) * 34;
        for (int b = 0; b < K / 32; ++b) {
            uint16_t s;
            memcpy(&s, p + 34 * b, 2);
            float scale = h2f(s);
            const int8_t *q = (const int8_t *)(p + 34 * b + 2);
            for (int i = 0; i < 32; ++i) {
                float v = scale * (float)q[i];
                dst[32 * b + i] = q8_round_half ? f16_round(v) : v;
            }
        }
        break;
    }
    case ORC_Q4_0: {
        /* GGUF Q4_0, dequantised by the reference's Q8_0 rule (cuda.cu:1104-1108):
         * w = (half)(float(d) * (nibble - 8)); byte i holds values i and i + 16 */
        const uint8_t *p = (const uint8_t *)w + row * (long)(K / 32) * 18;
        for (int b = 0; b < K / 32; ++b) {
            uint16_t s;
            memcpy(&s, p + 18 * b, 2);
            const float d = h2f(s);
            for (int i = 0; i < 16; ++i) {
                const uint8_t q = p[18 * b + 2 + i];
                const float v0 = d * (float)((int)(q & 15) - 8), v1 = d * (float)((int)(q >> 4) - 8);
                dst[32 * b + i] = q8_round_half ? f16_round(v0) : v0;
                dst[32 * b + 16 + i] = q8_round_half ? f16_round(v1) : v1;
            }
        }
        break;
    }
    default:
        abort();
    }
}

/* fp32 dot product with 8 independent partial sums (vectorisable without
 * reassociation flags); the partials are combined pairwise. */
inline float dot(const float *a, const float *b, int n) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int k = 0;
    for (; k + 8 <= n; k += 8)
        for (int j = 0; j < 8; ++j) acc[j] += a[k + j] * b[k + j];
    for (; k < n; ++k) acc[k & 7] += a[k] * b[k];
    return ((acc[0] + acc[4]) + (acc[1] + acc[5])) + ((acc[2] + acc[6]) + (acc[3] + acc[7]));
}

inline uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* Irwin-Hall(4) of 16-bit uniforms; integer exact so CPU and GPU agree bit for bit. */
inline float gen_one(uint64_t seed, uint64_t idx, float k) {
    uint64_t h = mix64(seed + (idx + 1) * 0x9E3779B97F4A7C15ull);
    int32_t s = (int32_t)(h & 0xffff) + (int32_t)((h >> 16) & 0xffff) +
                (int32_t)((h >> 32) & 0xffff) + (int32_t)((h >> 48) & 0xffff);
    return (float)(s - 131070) * k;
}

inline float gen_k(float stdv) { return stdv / 37837.227f; }

inline uint16_t f2h_bits(float x) {
    _Float16 h = (_Float16)x;
    uint16_t u;
    memcpy(&u, &h, 2);
    return u;
}

void quantize_block(const float *x, uint8_t *dst) {
    float amax = 0.f;
    for (int i = 0; i < 32; ++i) amax = std::max(amax, fabsf(x[i]));
    float d = amax / 127.0f;
    uint16_t s = f2h_bits(d);
    memcpy(dst, &s, 2);
    for (int i = 0; i < 32; ++i) {
        float q = d != 0.f ? roundf(x[i] / d) : 0.f;
        q = std::min(127.f, std::max(-127.f, q));
        dst[2 + i] = (uint8_t)(int8_t)q;
    }
}

/* ggml's Q4_0 quantisation (quantize_row_q4_0_reference, the published rule):
 * d = (value of largest magnitude, first occurrence) / -8, nibble =
 * min(15, (int)(x / d + 8.5)), byte i = nibble(x_i) | nibble(x_{i+16}) << 4. */
void quantize_block_q4_0(const float *x, uint8_t *dst) {
    float amax = 0.f, mx = 0.f;
    for (int i = 0; i < 32; ++i)
        if (fabsf(x[i]) > amax) {
            amax = fabsf(x[i]);
            mx = x[i];
        }
    const float d = mx / -8.0f;
    const float id = d != 0.f ? 1.0f / d : 0.f;
    uint16_t s = f2h_bits(d);
    memcpy(dst, &s, 2);
    for (int i = 0; i < 16; ++i) {
        const int n0 = std::min(15, (int)(x[i] * id + 8.5f));
        const int n1 = std::min(15, (int)(x[i + 16] * id + 8.5f));
        dst[2 + i] = (uint8_t)(n0 | (n1 << 4));
    }
}

}  // namespace

extern "C" {

float orc_round(int act, float x) { return rnd(act, x); }

void orc_round_array(int act, float *x, size_t n) {
    for (size_t i = 0; i < n; ++i) x[i] = rnd(act, x[i]);
}

void orc_f16_to_f32(const uint16_t *s, float *d, size_t n) {
    for (size_t i = 0; i < n; ++i) d[i] = h2f(s[i]);
}
void orc_f32_to_f16(const float *s, uint16_t *d, size_t n) {
    for (size_t i = 0; i < n; ++i) d[i] = f2h_bits(s[i]);
}
void orc_bf16_to_f32(const uint16_t *s, float *d, size_t n) {
    for (size_t i = 0; i < n; ++i) d[i] = b2f(s[i]);
}
void orc_f32_to_bf16(const float *s, uint16_t *d, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        float r = bf16_round(s[i]);
        uint32_t u;
        memcpy(&u, &r, 4);
        d[i] = (uint16_t)(u >> 16);
    }
}

int orc_num_threads(void) { return omp_get_max_threads(); }
void orc_set_f32_tf32(int on) { g_f32_tf32 = on; }
void orc_set_threads(int n) { omp_set_num_threads(n); }

void orc_gen_q4_0(uint8_t *out, int rows, int cols, uint64_t seed, float stdv) {
    const float k = gen_k(stdv);
#pragma omp parallel for schedule(static)
    for (long r = 0; r < rows; ++r) {
        float x[32];
        for (int b = 0; b < cols / 32; ++b) {
            const long blk = r * (cols / 32) + b;
            for (int i = 0; i < 32; ++i) x[i] = gen_one(seed, (uint64_t)(blk * 32 + i), k);
            quantize_block_q4_0(x, out + blk * 18);
        }
    }
}

void orc_quantize_q4_0(uint8_t *out, const float *x, int rows, int cols) {
    for (long b = 0; b < (long)rows * cols / 32; ++b) quantize_block_q4_0(x + b * 32, out + b * 18);
}

void orc_dequant_q4_0(float *out, const uint8_t *blocks, int rows, int cols, int out_half) {
#pragma omp parallel for schedule(static)
    for (long r = 0; r < rows; ++r) decode_row(blocks, ORC_Q4_0, r, cols, out + r * cols, out_half);
}

/* cuda.cu:389-421: out = (T)((float)scale * q) -- the fp32 product is exact. */
void orc_dequant_q8_0(float *out, const uint8_t *blocks, int rows, int cols, int out_half) {
#pragma omp parallel for schedule(static)
    for (long r = 0; r < rows; ++r) decode_row(blocks, ORC_Q8_0, r, cols, out + r * cols, out_half);
}

/* cuda.cu:1095-1111 (dispatch) + :270-341 (cuBLASLt): quantised weights are
 * dequantised to half first, then a T x T -> T GEMM with fp32 accumulation; the
 * bias epilogue adds before the final rounding. */
void orc_matmul(float *out, const float *x, const void *w, const float *bias, int M, int K, int N,
                int wtype, int act) {
    const bool tf = g_f32_tf32 && wtype == ORC_F32;
    std::vector<float> xt;
    if (tf) {
        xt.assign(x, x + (size_t)M * K);
        for (auto &v : xt) v = tf32_rn(v);
        x = xt.data();
    }
#pragma omp parallel
    {
        std::vector<float> row(K);
#pragma omp for schedule(static)
        for (long n = 0; n < N; ++n) {
            decode_row(w, wtype, n, K, row.data(), 1);
            if (tf)
                for (int k = 0; k < K; ++k) row[k] = tf32_rn(row[k]);
            for (long m = 0; m < M; ++m) {
                float acc = dot(x + m * K, row.data(), K);
                if (bias) acc += bias[n];
                out[m * N + n] = rnd(act, acc);
            }
        }
    }
}

/* cuda.cu:533-601: y = (x * rsqrt(mean(x^2) + eps)) * w, stored as T. */
void orc_rmsnorm(float *out, const float *x, const float *w, int rows, int C, float eps, int act) {
    for (long r = 0; r < rows; ++r) {
        const float *xr = x + r * C;
        float ss = dot(xr, xr, C);
        float mean = ss / (float)C;
        float s = 1.0f / sqrtf(mean + eps);
        for (int c = 0; c < C; ++c) out[r * C + c] = rnd(act, (xr[c] * s) * w[c]);
    }
}

/* cuda.cu:207-236: interleaved-pair rotation of the Q and K heads of each
 * [(NH + 2 kvNH) * HS] row; V is untouched.  Row r uses freqs[(pos0 + r) * HS]. */
void orc_rope_qkv(float *qkv, const float *freqs, int batch, int row, int pos0, int NH, int kvNH,
                  int HS, int act) {
    int W = (NH + 2 * kvNH) * HS;
    for (long b = 0; b < batch; ++b)
        for (int r = 0; r < row; ++r)
            for (int h = 0; h < NH + kvNH; ++h)
                for (int d = 0; d < HS / 2; ++d) {
                    const float *f = freqs + (long)(pos0 + r) * HS + 2 * d;
                    float c = f[0], s = f[1];
                    float *p = qkv + (b * row + r) * W + h * HS + 2 * d;
                    float xr = p[0], xi = p[1];
                    p[0] = rnd(act, xr * c - xi * s);
                    p[1] = rnd(act, xr * s + xi * c);
                }
}

/* cuda.h:15 declares cuda_rope (never defined by the reference): the same
 * rotation on a [batch, row, NH, HS] tensor. */
void orc_rope(float *x, const float *freqs, int batch, int row, int NH, int HS, int act) {
    for (long b = 0; b < batch; ++b)
        for (int r = 0; r < row; ++r)
            for (int h = 0; h < NH; ++h)
                for (int d = 0; d < HS / 2; ++d) {
                    const float *f = freqs + (long)r * HS + 2 * d;
                    float *p = x + ((b * row + r) * NH + h) * HS + 2 * d;
                    float xr = p[0], xi = p[1];
                    p[0] = rnd(act, xr * f[0] - xi * f[1]);
                    p[1] = rnd(act, xr * f[1] + xi * f[0]);
                }
}

/* cuda.cu:176-205: out = up * (gate * sigmoid(gate)), input row [up | gate]. */
void orc_swiglu(float *out, const float *inp, int rows, int C, int act) {
    std::vector<float> tmp((size_t)rows * C);
    for (long r = 0; r < rows; ++r)
        for (int c = 0; c < C; ++c) {
            float u = inp[r * 2 * C + c], g = inp[r * 2 * C + C + c];
            float sig = 1.0f / (1.0f + expf(-g));
            tmp[r * C + c] = rnd(act, (g * sig) * u);
        }
    memcpy(out, tmp.data(), sizeof(float) * tmp.size());
}

void orc_add(float *out, const float *a, const float *b, size_t n, int act) {
    for (size_t i = 0; i < n; ++i) out[i] = rnd(act, a[i] + b[i]);
}

void orc_div(float *out, const float *a, const float *b, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = a[i] / b[i];
}

/* cuda.cu:86-158: row softmax, exp(x - max) / sum. */
void orc_softmax(float *out, const float *inp, int rows, int cols) {
    for (long r = 0; r < rows; ++r) {
        const float *x = inp + r * cols;
        float m = -INFINITY;
        for (int i = 0; i < cols; ++i) m = fmaxf(m, x[i]);
        double sum = 0;
        std::vector<float> e(cols);
        for (int i = 0; i < cols; ++i) {
            e[i] = expf(x[i] - m);
            sum += e[i];
        }
        float inv = 1.0f / (float)sum;
        for (int i = 0; i < cols; ++i) out[r * cols + i] = e[i] * inv;
    }
}

/* One query row of the reference's causal attention (cuda.cu:767-852 with the
 * scaled softmax of :673-765): scores are stored as T, softmax numerators are
 * stored as T while their fp32 values are summed, probabilities are rounded to
 * T again after normalisation, and P.V is stored as T. */
static void attend_row(float *o, const float *q, const float *K, const float *V, long kstride,
                       int nkeys, int HS, int act, float *scratch) {
    const float scale = 1.0f / sqrtf((float)HS);
    float mx = -INFINITY;
    for (int j = 0; j < nkeys; ++j) {
        float s = rnd(act, dot(q, K + j * kstride, HS));
        scratch[j] = s;
        mx = fmaxf(mx, s * scale);
    }
    float sum = 0.f;
    for (int j = 0; j < nkeys; ++j) {
        float v = expf(scratch[j] * scale - mx);
        sum += v;
        scratch[j] = rnd(act, v);
    }
    float inv = 1.0f / sum;
    for (int j = 0; j < nkeys; ++j) scratch[j] = rnd(act, scratch[j] * inv);
    for (int d = 0; d < HS; ++d) {
        float acc = 0.f;
        for (int j = 0; j < nkeys; ++j) acc += scratch[j] * V[j * kstride + d];
        o[d] = rnd(act, acc);
    }
}

/* cuda.cu:1139-1145 (gq_sdpa) = repeat_qkv (:437-467) + mh_sdpa (:767-852). */
void orc_gqa_sdpa(float *out, const float *qkv, int batch, int row, int NH, int kvNH, int HS, int act) {
    int W = (NH + 2 * kvNH) * HS;
    int group = NH / kvNH;
#pragma omp parallel
    {
        std::vector<float> scratch(row);
#pragma omp for collapse(3) schedule(static)
        for (long b = 0; b < batch; ++b)
            for (int h = 0; h < NH; ++h)
                for (int i = 0; i < row; ++i) {
                    const float *base = qkv + b * row * W;
                    const float *q = base + (long)i * W + h * HS;
                    const float *K = base + NH * HS + (h / group) * HS;
                    const float *V = base + (NH + kvNH) * HS + (h / group) * HS;
                    attend_row(out + ((b * row + i) * NH + h) * HS, q, K, V, W, i + 1, HS, act,
                               scratch.data());
                }
    }
}

void orc_get_row(float *out, const float *inp, int batch, int row, int col, int idx) {
    if (idx < 0) idx += row;
    for (long b = 0; b < batch; ++b) memcpy(out + b * col, inp + (b * row + idx) * col, sizeof(float) * col);
}

/* cuda.cu:480-531 with block 256.  Thread tid scans packs tid, tid+256, ... with a
 * strict '>' (first occurrence wins); the shfl_down tree then prefers the lane
 * with the smaller bit-reversed index, and the cross-warp pass the warp with the
 * smaller bit-reversed index.  Elements past col/pack*pack are not scanned. */
static inline uint32_t brev5(uint32_t x) {
    uint32_t r = 0;
    for (int i = 0; i < 5; ++i) r |= ((x >> i) & 1u) << (4 - i);
    return r;
}

void orc_argmax(int *out, const float *inp, int rows, int cols, int pack) {
    int npack = cols / pack;
    for (long r = 0; r < rows; ++r) {
        const float *x = inp + r * cols;
        float best = -INFINITY;
        int bidx = -1;
        uint64_t bkey = ~0ull;
        for (int p = 0; p < npack; ++p)
            for (int e = 0; e < pack; ++e) {
                int idx = p * pack + e;
                float v = x[idx];
                uint32_t tid = p % 256, j = p / 256;
                uint64_t key = ((uint64_t)brev5(tid / 32) << 58) | ((uint64_t)brev5(tid % 32) << 53) |
                               ((uint64_t)j << 8) | (uint64_t)e;
                if (v > best || (v == best && bidx >= 0 && key < bkey)) {
                    best = v;
                    bidx = idx;
                    bkey = key;
                }
            }
        out[r] = bidx;
    }
}

/* Sampling beyond argmax.  The reference has none (cuda.cu:988 leaves it as a
 * TODO), so this restates the library's published rule, not reference code:
 * candidates = the min(top_k, 256) largest values (top_k <= 0: 256), ties by
 * smaller index; e_i = exp((l_i - l_max) / temperature); prefix sums c_i; the
 * shortest prefix m with c_m >= top_p * c_K (top_p outside (0, 1): all K);
 * u = (top 24 bits of mix64(seed + 0x9E3779B97F4A7C15 * (step * 65536 + row + 1)))
 * * 2^-24 * c_m; the token is the first candidate with c_i > u.  u_out (may be
 * null) receives u / c_m and the relative distance of u to the nearest
 * prefix-sum boundary, for tolerance checks. */
void orc_sample(int *out, float *u_out, const float *logits, int rows, int V, float temperature, int top_k,
                float top_p, uint64_t seed, const int64_t *steps) {
    for (int r = 0; r < rows; ++r) {
        const float *x = logits + (size_t)r * V;
        const int K = std::min(top_k > 0 && top_k < 256 ? top_k : 256, V);
        std::vector<int> idx(V);
        for (int i = 0; i < V; ++i) idx[i] = i;
        std::partial_sort(idx.begin(), idx.begin() + K, idx.end(),
                          [&](int a, int b) { return x[a] > x[b] || (x[a] == x[b] && a < b); });
        std::vector<float> c(K);
        const float lmax = x[idx[0]], invt = 1.0f / temperature;
        float run = 0.f;
        for (int i = 0; i < K; ++i) {
            run += expf((x[idx[i]] - lmax) * invt);
            c[i] = run;
        }
        int m = K;
        if (top_p > 0.f && top_p < 1.f) {
            const float target = top_p * run;
            for (int i = 0; i < K; ++i)
                if (c[i] >= target) {
                    m = i + 1;
                    break;
                }
        }
        const uint64_t h = mix64(seed + 0x9E3779B97F4A7C15ull * (uint64_t)(steps[r] * 65536 + r + 1));
        const float frac = (float)(h >> 40) * (1.0f / 16777216.0f);
        const float u = frac * c[m - 1];
        int pick = m - 1;
        for (int i = 0; i < m; ++i)
            if (c[i] > u) {
                pick = i;
                break;
            }
        out[r] = idx[pick];
        if (u_out) {
            float dist = INFINITY;
            for (int i = 0; i < m; ++i) dist = std::min(dist, fabsf(c[i] - u) / c[m - 1]);
            u_out[2 * r] = frac;
            u_out[2 * r + 1] = dist;
        }
    }
}

/* cuda.cu:1232-1255: row gather; quantised tables are dequantised to half. */
void orc_embedding(float *out, const int *ids, const void *table, int n, int col, int dtype) {
    for (long i = 0; i < n; ++i) decode_row(table, dtype, ids[i], col, out + i * col, 1);
}

/* cuda.cu:902-926: rmsnorm -> qkv matmul -> rope -> causal GQA sdpa -> o matmul -> residual. */
void orc_gqa_layer(float *x, const float *freqs, const float *norm_w, const void *qkv_w, const void *out_w,
                   int B, int n, int pos0, int NH, int kvNH, int HS, float eps, int wtype, int act,
                   float *kcache, float *vcache, int cap) {
    int d = NH * HS, W = (NH + 2 * kvNH) * HS, group = NH / kvNH;
    long rows = (long)B * n;
    std::vector<float> a(rows * d), qkv(rows * W), att(rows * d), o(rows * d);
    orc_rmsnorm(a.data(), x, norm_w, rows, d, eps, act);
    orc_matmul(qkv.data(), a.data(), qkv_w, nullptr, rows, d, W, wtype, act);
    orc_rope_qkv(qkv.data(), freqs, B, n, pos0, NH, kvNH, HS, act);
    for (long b = 0; b < B; ++b)
        for (int i = 0; i < n; ++i)
            for (int h = 0; h < kvNH; ++h) {
                const float *src = qkv.data() + (b * n + i) * W;
                long dst = ((b * kvNH + h) * cap + pos0 + i) * HS;
                memcpy(kcache + dst, src + d + h * HS, sizeof(float) * HS);
                memcpy(vcache + dst, src + d + kvNH * HS + h * HS, sizeof(float) * HS);
            }
#pragma omp parallel
    {
        std::vector<float> scratch(pos0 + n);
#pragma omp for collapse(3) schedule(static)
        for (long b = 0; b < B; ++b)
            for (int h = 0; h < NH; ++h)
                for (int i = 0; i < n; ++i) {
                    const float *q = qkv.data() + (b * n + i) * W + h * HS;
                    const float *K = kcache + (b * kvNH + h / group) * (long)cap * HS;
                    const float *V = vcache + (b * kvNH + h / group) * (long)cap * HS;
                    attend_row(att.data() + (b * n + i) * d + h * HS, q, K, V, HS, pos0 + i + 1, HS, act,
                               scratch.data());
                }
    }
    orc_matmul(o.data(), att.data(), out_w, nullptr, rows, d, d, wtype, act);
    orc_add(x, x, o.data(), rows * d, act);
}

/* cuda.cu:928-945: rmsnorm -> fc ([up|gate]) matmul -> swiglu -> down matmul -> residual. */
void orc_ffn_layer(float *x, const float *norm_w, const void *fc_w, const void *down_w, int B, int n, int d,
                   int F, float eps, int wtype, int act) {
    long rows = (long)B * n;
    std::vector<float> a(rows * d), fc(rows * 2 * F), h(rows * F), o(rows * d);
    orc_rmsnorm(a.data(), x, norm_w, rows, d, eps, act);
    orc_matmul(fc.data(), a.data(), fc_w, nullptr, rows, d, 2 * F, wtype, act);
    orc_swiglu(h.data(), fc.data(), rows, F, act);
    orc_matmul(o.data(), h.data(), down_w, nullptr, rows, F, d, wtype, act);
    orc_add(x, x, o.data(), rows * d, act);
}

/* cuda.cu:975-981: last row of each batch -> rmsnorm -> logits matmul. */
void orc_classify(float *logits, const float *x, const float *norm_w, const void *w, int B, int T, int d,
                  int V, float eps, int wtype, int act) {
    std::vector<float> last((size_t)B * d), a((size_t)B * d);
    orc_get_row(last.data(), x, B, T, d, -1);
    orc_rmsnorm(a.data(), last.data(), norm_w, B, d, eps, act);
    orc_matmul(logits, a.data(), w, nullptr, B, d, V, wtype, act);
}

void orc_gen_normal(float *dst, size_t n, uint64_t seed, float stdv) {
    float k = gen_k(stdv);
#pragma omp parallel for schedule(static)
    for (long i = 0; i < (long)n; ++i) dst[i] = gen_one(seed, (uint64_t)i, k);
}

void orc_gen_f16(uint16_t *dst, size_t n, uint64_t seed, float stdv) {
    float k = gen_k(stdv);
#pragma omp parallel for schedule(static)
    for (long i = 0; i < (long)n; ++i) dst[i] = f2h_bits(gen_one(seed, (uint64_t)i, k));
}

void orc_gen_q8_0(uint8_t *dst, int rows, int cols, uint64_t seed, float stdv) {
    float k = gen_k(stdv);
    long nb = cols / 32;
#pragma omp parallel for schedule(static)
    for (long blk = 0; blk < (long)rows * nb; ++blk) {
        float x[32];
        for (int i = 0; i < 32; ++i) x[i] = gen_one(seed, (uint64_t)(blk * 32 + i), k);
        quantize_block(x, dst + blk * 34);
    }
}

void orc_quantize_q8_0(uint8_t *dst, const float *src, int rows, int cols) {
    long nb = cols / 32;
    for (long blk = 0; blk < (long)rows * nb; ++blk) quantize_block(src + blk * 32, dst + blk * 34);
}

/* llama.go:54-67: freq = 1 / float32(pow(theta, 2i/HS)) / factor[i];
 * angle = float32(j) * freq; table = (cos, sin) of the float32 angle. */
void orc_make_freqs(float *out, const float *factor, int HS, int ctx, float theta) {
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

}  // extern "C"
