// Tensor parallelism inside one node, one process per GPU (Megatron-style):
// column-parallel q|k|v and up|gate, row-parallel o and down (each rank holds a
// K-slice and produces fp32 partial sums), vocabulary-parallel logits.
//
// Exchanges per layer: one all-reduce of the fp32 partials after o and one
// after down ([rows, d] fp32), followed by the residual add with the
// reference's rounding (y = T(sum of partials), x = T(x + y): the same formula
// as the single-GPU RESID epilogue, cuda.cu:423-435 after :1095-1111, up to
// the fp32 summation order).  The logits head exchanges one (value, order key)
// winner per row and rank and picks the best with the reference argmax's tie
// order (cuda.cu:480-531), so the token equals the single-GPU token.
//
// The collectives are NCCL's, loaded at run time (dlopen of libnccl.so.2) so
// that the library still links with the reference's cgo line
// (-lcublasLt -lcudart -lm -lcublas) and hosts without NCCL are unaffected.
#include <dlfcn.h>
#include <nccl.h>  // types only; every function is resolved with dlsym
#include <string.h>

#include <vector>

#include "common.cuh"
#include "wukong_ext.h"
#include "wukong_internal.cuh"

namespace wk {

namespace {

struct NcclApi {
    void *handle = nullptr;
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char *(*error_string)(ncclResult_t) = nullptr;
};
NcclApi g_nccl;
ncclComm_t g_comm = nullptr;
int g_rank = 0, g_world = 1;

int load_nccl() {
    if (g_nccl.handle) return 0;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return fail("tensor parallelism needs NCCL: dlopen(libnccl.so.2) failed: %s", dlerror());
    NcclApi a;
    a.handle = h;
#define WK_NCCL_SYM(field, name)                                           \
    a.field = (decltype(a.field))dlsym(h, name);                          \
    if (!a.field) return fail("libnccl.so.2 does not export %s", name);
    WK_NCCL_SYM(get_unique_id, "ncclGetUniqueId")
    WK_NCCL_SYM(comm_init_rank, "ncclCommInitRank")
    WK_NCCL_SYM(comm_destroy, "ncclCommDestroy")
    WK_NCCL_SYM(all_reduce, "ncclAllReduce")
    WK_NCCL_SYM(all_gather, "ncclAllGather")
    WK_NCCL_SYM(error_string, "ncclGetErrorString")
#undef WK_NCCL_SYM
    g_nccl = a;
    return 0;
}

void nccl_check(ncclResult_t r, const char *what) {
    if (r != ncclSuccess) WK_PANIC("%s failed: %s", what, g_nccl.error_string ? g_nccl.error_string(r) : "?");
}

// x = T(x + T(p)): the residual add of a row-parallel layer after its all-reduce
template <typename T> __global__ void resid_from_partial_kernel(T *__restrict__ x, const float *__restrict__ p, long n) {
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[i] = from_float<T>(to_float(x[i]) + round_to<T>(p[i]));
}

// rec: [world][chunk bytes] with, per rank, keys [B] (u64) then values [B] (f32)
__global__ void argmax_combine_kernel(int *__restrict__ tokens, const uint8_t *__restrict__ rec, long chunk, int B,
                                      int world, int pack) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    float bv = -INFINITY;
    uint64_t bk = ~0ull;
    for (int r = 0; r < world; ++r) {
        const uint64_t k = reinterpret_cast<const uint64_t *>(rec + r * chunk)[b];
        const float v = reinterpret_cast<const float *>(rec + r * chunk + 8L * B)[b];
        if (k == ~0ull) continue;
        if (v > bv || (v == bv && k < bk)) {
            bv = v;
            bk = k;
        }
    }
    tokens[b] = logits_index(bk, pack);
}

// ---------------------------------------------------------------- one-shot exchange over peer memory
// Each rank exports one buffer (CUDA IPC, layout kX* in wukong_internal.cuh)
// that all ranks map.  A rank writes its payload into its own slot, publishes
// the epoch in its own flag (release, system scope), waits (bounded) for every
// peer's flag, and reads the peers' slots directly over NVLink (plain loads,
// no multicast).  Payload slots alternate by epoch parity: a rank reuses a
// slot two calls later, when every peer has already published its next call,
// which it does only after it has finished reading this one.
//   all-reduce kernel (rows beyond one decode GEMV): flags [2][16 CTAs],
//   logits winners: flags [2], decode ARESID GEMV tiles: one flag per tile.
constexpr int kArCtas = 16;
constexpr size_t kArSlot = kXArSlot;
constexpr size_t kWinSlot = kXWinSlot;
constexpr size_t kP2POff = kXArPay;
constexpr size_t kP2PBytes = kXBytes;
constexpr int kMaxWorld = 8;
static_assert(kXArPay + 2 * kXArSlot == kXWinPay && kMaxWorld == kTpMaxWorld, "exchange layout");

struct P2P {
    bool ok = false;
    uint8_t *mine = nullptr;              // this rank's exported buffer
    uint8_t *peers_h[kMaxWorld] = {};     // mapped buffers of all ranks (own included)
    uint8_t **peers_d = nullptr;          // the same, on the device
    unsigned long long *epochs = nullptr; // call counters: [kArCtas] all-reduce CTAs, [1] winners, [kTpMaxTiles] tiles
};
P2P g_p2p;

// x = T(x + T(sum over ranks of partial)) for n values; CTA c owns values [c n/k, (c+1) n/k).
template <typename T>
__global__ void __launch_bounds__(512) p2p_allreduce_resid_kernel(T *__restrict__ x, const float *__restrict__ partial,
                                                                  long n, uint8_t *const *peers, int rank, int world,
                                                                  unsigned long long *epochs, int *err,
                                                                  unsigned long long limit_ns) {
    __shared__ unsigned long long e_s;
    __shared__ int ok_s;
    const int c = blockIdx.x, tid = threadIdx.x;
    const long per = (n + gridDim.x - 1) / gridDim.x;
    const long lo = c * per, hi = min(n, lo + per);
    if (tid == 0) {
        e_s = ++epochs[c];
        ok_s = 1;
    }
    __syncthreads();
    const unsigned long long e = e_s;
    const int par = (int)(e & 1);
    float *mine = reinterpret_cast<float *>(peers[rank] + kP2POff + par * kArSlot);
    for (long i = lo + tid; i < hi; i += blockDim.x) mine[i] = partial[i];
    __syncthreads();
    if (tid == 0) {
        __threadfence_system();
        st_release_sys(reinterpret_cast<unsigned long long *>(peers[rank]) + par * kArCtas + c, e);
    }
    if (tid < world && !wait_flag(reinterpret_cast<const unsigned long long *>(peers[tid]) + par * kArCtas + c, e,
                                  err, 40, limit_ns))
        ok_s = 0;
    __syncthreads();
    if (!ok_s) return;
    for (long i = lo + tid; i < hi; i += blockDim.x) {
        float acc = 0.f;
        for (int r = 0; r < world; ++r)
            acc += __ldcv(reinterpret_cast<const float *>(peers[r] + kP2POff + par * kArSlot) + i);
        x[i] = from_float<T>(to_float(x[i]) + round_to<T>(acc));
    }
}

// Logits winners: keys [B] u64 and values [B] f32 of every rank -> token ids.
__global__ void __launch_bounds__(32) p2p_argmax_kernel(int *__restrict__ tokens, const uint8_t *__restrict__ send, int B,
                                                        int pack, uint8_t *const *peers, int rank, int world,
                                                        unsigned long long *epochs, int *err,
                                                        unsigned long long limit_ns) {
    __shared__ unsigned long long e_s;
    __shared__ int ok_s;
    const int tid = threadIdx.x;
    const size_t bytes = ((size_t)B * 12 + 15) / 16 * 16;  // keys [B] u64, then values [B] f32
    if (tid == 0) {
        e_s = ++epochs[kArCtas];
        ok_s = 1;
    }
    __syncthreads();
    const unsigned long long e = e_s;
    const int par = (int)(e & 1);
    uint8_t *mine = peers[rank] + kP2POff + 2 * kArSlot + par * kWinSlot;
    for (size_t i = tid * 4; i < bytes; i += 32 * 4)
        *reinterpret_cast<uint32_t *>(mine + i) = *reinterpret_cast<const uint32_t *>(send + i);
    __syncthreads();
    if (tid == 0) {
        __threadfence_system();
        st_release_sys(reinterpret_cast<unsigned long long *>(peers[rank] + 256) + par, e);
    }
    if (tid < world &&
        !wait_flag(reinterpret_cast<const unsigned long long *>(peers[tid] + 256) + par, e, err, 41, limit_ns))
        ok_s = 0;
    __syncthreads();
    if (!ok_s) return;
    for (int b = tid; b < B; b += 32) {
        float bv = -INFINITY;
        uint64_t bk = ~0ull;
        for (int r = 0; r < world; ++r) {
            const uint8_t *rec = peers[r] + kP2POff + 2 * kArSlot + par * kWinSlot;
            const uint64_t k = __ldcv(reinterpret_cast<const unsigned long long *>(rec) + b);
            const float v = __ldcv(reinterpret_cast<const float *>(rec + 8L * B) + b);
            if (k == ~0ull) continue;
            if (v > bv || (v == bv && k < bk)) {
                bv = v;
                bk = k;
            }
        }
        tokens[b] = logits_index(bk, pack);
    }
}

// Map every rank's exchange buffer (collective: all ranks call it after the
// communicator exists).  Returns false on every rank if any rank failed.
bool p2p_setup() {
    bool ok = g_world <= kMaxWorld;
    const char *env = getenv("WUKONG_TP_P2P");
    if (env && env[0] == '0') ok = false;
    cudaIpcMemHandle_t mine_h = {};
    if (ok) ok = cudaMalloc(&g_p2p.mine, kP2PBytes) == cudaSuccess &&
                 cudaMemset(g_p2p.mine, 0, kP2PBytes) == cudaSuccess &&
                 cudaIpcGetMemHandle(&mine_h, g_p2p.mine) == cudaSuccess;
    // exchange handles (and the local verdict) through the communicator
    struct Rec {
        cudaIpcMemHandle_t h;
        int ok;
        int pad[15];
    };
    Rec rec = {};
    rec.h = mine_h;
    rec.ok = ok ? 1 : 0;
    Rec *d = nullptr;
    Rec *all = (Rec *)calloc(g_world, sizeof(Rec));
    cudaStream_t s = stream();
    WK_CHECK(cudaMalloc(&d, sizeof(Rec) * (g_world + 1)));
    WK_CHECK(cudaMemcpy(d + g_world, &rec, sizeof(Rec), cudaMemcpyHostToDevice));
    nccl_check(g_nccl.all_gather(d + g_world, d, sizeof(Rec), ncclUint8, g_comm, s), "ncclAllGather");
    WK_CHECK(cudaStreamSynchronize(s));
    WK_CHECK(cudaMemcpy(all, d, sizeof(Rec) * g_world, cudaMemcpyDeviceToHost));
    cudaFree(d);
    for (int r = 0; r < g_world; ++r) ok = ok && all[r].ok;
    for (int r = 0; ok && r < g_world; ++r) {
        if (r == g_rank) {
            g_p2p.peers_h[r] = g_p2p.mine;
            continue;
        }
        void *pp = nullptr;
        ok = cudaIpcOpenMemHandle(&pp, all[r].h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
        g_p2p.peers_h[r] = (uint8_t *)pp;
    }
    free(all);
    // every rank must agree before any kernel relies on the mappings
    int *flag = nullptr;
    int v = ok ? 1 : 0;
    WK_CHECK(cudaMalloc(&flag, sizeof(int)));
    WK_CHECK(cudaMemcpy(flag, &v, sizeof(int), cudaMemcpyHostToDevice));
    nccl_check(g_nccl.all_reduce(flag, flag, 1, ncclInt32, ncclMin, g_comm, s), "ncclAllReduce");
    WK_CHECK(cudaStreamSynchronize(s));
    WK_CHECK(cudaMemcpy(&v, flag, sizeof(int), cudaMemcpyDeviceToHost));
    cudaFree(flag);
    ok = v == 1;
    if (ok) ok = cudaMalloc(&g_p2p.peers_d, sizeof(uint8_t *) * kMaxWorld) == cudaSuccess &&
                 cudaMemcpy(g_p2p.peers_d, g_p2p.peers_h, sizeof(uint8_t *) * kMaxWorld, cudaMemcpyHostToDevice) ==
                     cudaSuccess &&
                 cudaMalloc(&g_p2p.epochs, sizeof(unsigned long long) * (kArCtas + 1 + kTpMaxTiles)) == cudaSuccess &&
                 cudaMemset(g_p2p.epochs, 0, sizeof(unsigned long long) * (kArCtas + 1 + kTpMaxTiles)) == cudaSuccess;
    cudaGetLastError();
    g_p2p.ok = ok;
    return ok;
}

void p2p_teardown() {
    for (int r = 0; r < kMaxWorld; ++r)
        if (g_p2p.peers_h[r] && g_p2p.peers_h[r] != g_p2p.mine) cudaIpcCloseMemHandle(g_p2p.peers_h[r]);
    if (g_p2p.mine) cudaFree(g_p2p.mine);
    if (g_p2p.peers_d) cudaFree(g_p2p.peers_d);
    if (g_p2p.epochs) cudaFree(g_p2p.epochs);
    g_p2p = P2P();
}

}  // namespace

bool tp_active() { return g_comm != nullptr && g_world > 1; }

bool tp_link(TpLink *link) {
    if (!g_p2p.ok || !tp_active()) return false;
    link->peers = g_p2p.peers_d;
    link->rank = g_rank;
    link->world = g_world;
    link->win_epoch = g_p2p.epochs + kArCtas;
    link->tile_epoch = g_p2p.epochs + kArCtas + 1;
    link->limit_ns = g_rt.wait_limit_ns;
    return true;
}
int tp_rank() { return g_rank; }
int tp_world() { return g_world; }

void tp_allreduce_f32(float *buf, size_t n, cudaStream_t s) {
    nccl_check(g_nccl.all_reduce(buf, buf, n, ncclFloat32, ncclSum, g_comm, s), "ncclAllReduce");
}

size_t tp_winner_chunk(int B) { return ((size_t)B * 12 + 15) / 16 * 16; }

void tp_argmax_combine(int *tokens, const void *send, void *recv, int B, int pack, cudaStream_t s) {
    const size_t chunk = tp_winner_chunk(B);
    if (g_p2p.ok && chunk <= kWinSlot) {
        p2p_argmax_kernel<<<1, 32, 0, s>>>(tokens, (const uint8_t *)send, B, pack, g_p2p.peers_d, g_rank, g_world,
                                           g_p2p.epochs, g_rt.d_error, g_rt.wait_limit_ns);
        WK_CHECK_LAUNCH();
        return;
    }
    nccl_check(g_nccl.all_gather(send, recv, chunk, ncclUint8, g_comm, s), "ncclAllGather");
    argmax_combine_kernel<<<(B + 127) / 128, 128, 0, s>>>(tokens, (const uint8_t *)recv, (long)chunk, B, g_world,
                                                         pack);
    WK_CHECK_LAUNCH();
}

template <typename T> int allreduce_resid(T *x, float *p, long n, cudaStream_t s) {
    if (n <= 0) return 0;
    if (g_p2p.ok && (size_t)n * sizeof(float) <= kArSlot) {
        // always kArCtas CTAs: every CTA index takes part in every call, so all
        // CTAs of a call use the same slot parity (see the layout comment)
        p2p_allreduce_resid_kernel<T><<<kArCtas, 512, 0, s>>>(x, p, n, g_p2p.peers_d, g_rank, g_world, g_p2p.epochs,
                                                           g_rt.d_error, g_rt.wait_limit_ns);
        WK_CHECK_LAUNCH();
        return 1;
    }
    tp_allreduce_f32(p, (size_t)n, s);
    resid_from_partial<T>(x, p, n, s);
    return 1;
}
template int allreduce_resid<__half>(__half *, float *, long, cudaStream_t);
template int allreduce_resid<__nv_bfloat16>(__nv_bfloat16 *, float *, long, cudaStream_t);

template <typename T> void resid_from_partial(T *x, const float *p, long n, cudaStream_t s) {
    if (n <= 0) return;
    resid_from_partial_kernel<T><<<(unsigned)((n + 255) / 256), 256, 0, s>>>(x, p, n);
    WK_CHECK_LAUNCH();
}
template void resid_from_partial<__half>(__half *, const float *, long, cudaStream_t);
template void resid_from_partial<__nv_bfloat16>(__nv_bfloat16 *, const float *, long, cudaStream_t);

}  // namespace wk

using namespace wk;

extern "C" {

int wk_tp_unique_id(void *id) {
    if (!id) return fail("wk_tp_unique_id: null buffer");
    if (load_nccl()) return -1;
    ncclUniqueId u;
    ncclResult_t r = g_nccl.get_unique_id(&u);
    if (r != ncclSuccess) return fail("ncclGetUniqueId: %s", g_nccl.error_string(r));
    memcpy(id, &u, sizeof(u));
    return 0;
}

int wk_tp_init(int rank, int world, const void *id) {
    if (world < 1 || rank < 0 || rank >= world || !id) return fail("wk_tp_init: bad rank %d / world %d", rank, world);
    if (g_rt.device < 0) return fail("wk_tp_init: cuda_init() has not been called");
    if (g_comm) return fail("wk_tp_init: already initialised (call wk_tp_fini first)");
    if (load_nccl()) return -1;
    set_device_current();
    ncclUniqueId u;
    memcpy(&u, id, sizeof(u));
    ncclResult_t r = g_nccl.comm_init_rank(&g_comm, world, u, rank);
    if (r != ncclSuccess) {
        g_comm = nullptr;
        return fail("ncclCommInitRank(rank %d of %d): %s", rank, world, g_nccl.error_string(r));
    }
    g_rank = rank;
    g_world = world;
    p2p_setup();  // the one-shot exchange over peer memory, or NCCL if any rank cannot map the others
    return 0;
}

void wk_tp_fini(void) {
    if (g_comm) {
        cudaStreamSynchronize(stream());
        p2p_teardown();
        g_nccl.comm_destroy(g_comm);
    }
    g_comm = nullptr;
    g_rank = 0;
    g_world = 1;
}

int wk_tp_exchange_selftest(int world, int publish) {
    if (g_rt.device < 0) return fail("wk_tp_exchange_selftest: cuda_init() has not been called");
    if (world < 2 || world > kMaxWorld) return fail("wk_tp_exchange_selftest: world %d outside [2, %d]", world, kMaxWorld);
    set_device_current();
    cudaStream_t s = stream();
    const long n = 4096;  // one decode row of an 8B model
    uint8_t *bufs[kMaxWorld] = {};
    uint8_t **peers_d = nullptr;
    unsigned long long *epochs = nullptr;
    __half *x = nullptr;
    float *partial = nullptr;
    int rc = 0;
    auto ok = [&](cudaError_t e) {
        if (e != cudaSuccess && rc == 0) rc = fail("wk_tp_exchange_selftest: %s", cudaGetErrorString(e));
        return rc == 0;
    };
    for (int r = 0; r < world && ok(cudaMalloc(&bufs[r], kP2PBytes)); ++r) ok(cudaMemset(bufs[r], 0, kP2PBytes));
    ok(cudaMalloc(&peers_d, sizeof(uint8_t *) * kMaxWorld)) &&
        ok(cudaMemcpy(peers_d, bufs, sizeof(uint8_t *) * kMaxWorld, cudaMemcpyHostToDevice));
    ok(cudaMalloc(&epochs, sizeof(unsigned long long) * (kArCtas + 1))) &&
        ok(cudaMemset(epochs, 0, sizeof(unsigned long long) * (kArCtas + 1)));
    ok(cudaMalloc(&x, sizeof(__half) * n)) && ok(cudaMalloc(&partial, sizeof(float) * n));
    if (rc == 0) {
        std::vector<__half> hx(n, __float2half(1.0f));
        std::vector<float> hp(n, 1.0f);
        ok(cudaMemcpy(x, hx.data(), sizeof(__half) * n, cudaMemcpyHostToDevice));
        ok(cudaMemcpy(partial, hp.data(), sizeof(float) * n, cudaMemcpyHostToDevice));
        if (publish) {
            // the emulated ranks' first call (epoch 1, slot parity 1): partials of 1.0 and every CTA's flag
            std::vector<unsigned long long> flags(kArCtas, 1ull);
            for (int r = 1; r < world; ++r) {
                ok(cudaMemcpy(bufs[r] + kP2POff + kArSlot, hp.data(), sizeof(float) * n, cudaMemcpyHostToDevice));
                ok(cudaMemcpy(reinterpret_cast<unsigned long long *>(bufs[r]) + kArCtas, flags.data(),
                              sizeof(unsigned long long) * kArCtas, cudaMemcpyHostToDevice));
            }
        }
    }
    if (rc == 0) {
        ok(cudaStreamSynchronize(s));
        p2p_allreduce_resid_kernel<__half><<<kArCtas, 512, 0, s>>>(x, partial, n, peers_d, 0, world, epochs,
                                                                g_rt.d_error, g_rt.wait_limit_ns);
        ok(cudaGetLastError()) && ok(cudaStreamSynchronize(s));
    }
    if (rc == 0) {
        rc = *(volatile int *)g_rt.h_error;
        if (rc == 0) {
            // x = T(1 + T(world * 1.0))
            std::vector<__half> hx(n);
            ok(cudaMemcpy(hx.data(), x, sizeof(__half) * n, cudaMemcpyDeviceToHost));
            for (long i = 0; rc == 0 && i < n; ++i)
                if (__half2float(hx[i]) != 1.0f + (float)world) rc = -2;
            if (rc == -2) fail("wk_tp_exchange_selftest: wrong sum");
        }
    }
    for (int r = 0; r < world; ++r)
        if (bufs[r]) cudaFree(bufs[r]);
    for (void *p : {(void *)peers_d, (void *)epochs, (void *)x, (void *)partial})
        if (p) cudaFree(p);
    return rc;
}

int wk_tp_gemv_selftest(int world, int N, int K, int M) {
    if (g_rt.device < 0) return fail("wk_tp_gemv_selftest: cuda_init() has not been called");
    if (world < 2 || world > kMaxWorld || M < 1 || M > 8 || K % 256 || N % 16 || N / 16 > kTpMaxTiles)
        return fail("wk_tp_gemv_selftest: world %d, N %d, K %d, M %d not supported", world, N, K, M);
    set_device_current();
    cudaStream_t s = stream();
    const size_t wbytes = (size_t)N * (K / 32) * 34;
    uint8_t *bufs[kMaxWorld] = {};
    uint8_t **peers_d = nullptr;
    unsigned long long *epochs = nullptr;
    void *w = nullptr, *x = nullptr, *res = nullptr;
    float *p32 = nullptr;
    int rc = 0;
    auto ok = [&](cudaError_t e) {
        if (e != cudaSuccess && rc == 0) rc = fail("wk_tp_gemv_selftest: %s", cudaGetErrorString(e));
        return rc == 0;
    };
    for (int r = 0; r < world && ok(cudaMalloc(&bufs[r], kP2PBytes)); ++r) ok(cudaMemset(bufs[r], 0, kP2PBytes));
    ok(cudaMalloc(&peers_d, sizeof(uint8_t *) * kMaxWorld)) &&
        ok(cudaMemcpy(peers_d, bufs, sizeof(uint8_t *) * kMaxWorld, cudaMemcpyHostToDevice));
    ok(cudaMalloc(&epochs, sizeof(unsigned long long) * (1 + kTpMaxTiles))) &&
        ok(cudaMemset(epochs, 0, sizeof(unsigned long long) * (1 + kTpMaxTiles)));
    ok(cudaMalloc(&w, wbytes)) && ok(cudaMalloc(&x, 2 * (size_t)M * K)) && ok(cudaMalloc(&res, 2 * (size_t)M * N)) &&
        ok(cudaMalloc(&p32, 4 * (size_t)M * N));
    if (rc == 0 && (wk_fill_random_q8_0(w, N, K, 101, 0.02f) || wk_fill_random_f16(x, (long)M * K, 102, 1.0f) ||
                    wk_fill_random_f16(res, (long)M * N, 103, 1.0f)))
        rc = -1;
    // the emulated ranks q = 1..world-1 pushed every tile of their first call (epoch 1,
    // slot parity 1) to rank 0, with the partial sums 0.25 q
    if (rc == 0) {
        std::vector<unsigned long long> words((size_t)N / 16 * kTpMaxWorld * 128, 0ull);
        for (int t = 0; t < N / 16; ++t)
            for (int q = 1; q < world; ++q)
                for (int i = 0; i < 128; ++i) {
                    const float v = 0.25f * q;
                    uint32_t bits;
                    memcpy(&bits, &v, 4);
                    words[((size_t)t * kTpMaxWorld + q) * 128 + i] = (1ull << 32) | bits;
                }
        ok(cudaMemcpy(bufs[0] + kXTileLL + (size_t)kTpMaxTiles * kTpMaxWorld * 128 * 8, words.data(), words.size() * 8,
                      cudaMemcpyHostToDevice));
    }
    std::vector<__half> h_res((size_t)M * N), h_out((size_t)M * N);
    std::vector<float> h_p((size_t)M * N);
    if (rc == 0) ok(cudaMemcpy(h_res.data(), res, 2 * (size_t)M * N, cudaMemcpyDeviceToHost));
    if (rc == 0) {
        GemvArgs a;
        a.w = (const uint8_t *)w;
        a.wtype = kQ8_0;
        a.N = N;
        a.K = K;
        a.x = x;
        a.ldx = K;
        a.M = M;
        a.epi = EPI_PARTIAL;
        a.out = p32;
        a.ldo = N;
        gemv(a, kF16, s);  // this rank's partial sums, for the check
        GemvArgs b = a;
        b.epi = EPI_ARESID;
        b.out = res;
        b.res = res;
        b.ldr = N;
        b.tp.peers = peers_d;
        b.tp.rank = 0;
        b.tp.world = world;
        b.tp.win_epoch = epochs;
        b.tp.tile_epoch = epochs + 1;
        b.tp.limit_ns = g_rt.wait_limit_ns;
        gemv(b, kF16, s);
        ok(cudaStreamSynchronize(s));
    }
    if (rc == 0) rc = *(volatile int *)g_rt.h_error;
    if (rc == 0) {
        ok(cudaMemcpy(h_p.data(), p32, 4 * (size_t)M * N, cudaMemcpyDeviceToHost));
        ok(cudaMemcpy(h_out.data(), res, 2 * (size_t)M * N, cudaMemcpyDeviceToHost));
        for (size_t i = 0; rc == 0 && i < h_out.size(); ++i) {
            float acc = 0.f;
            acc += h_p[i];
            for (int q = 1; q < world; ++q) acc += 0.25f * q;
            const float want = __half2float(__float2half(__half2float(h_res[i]) + __half2float(__float2half(acc))));
            if (__half2float(h_out[i]) != want) rc = fail("wk_tp_gemv_selftest: element %zu is %g, expected %g", i,
                                                         (double)__half2float(h_out[i]), (double)want) - 1;
        }
    }
    for (int r = 0; r < world; ++r)
        if (bufs[r]) cudaFree(bufs[r]);
    for (void *p : {(void *)peers_d, (void *)epochs, w, x, res, (void *)p32})
        if (p) cudaFree(p);
    return rc;
}

int wk_tp_rank(void) { return g_rank; }
int wk_tp_world(void) { return g_world; }
int wk_tp_p2p(void) { return g_p2p.ok ? 1 : 0; }

}  // extern "C"
