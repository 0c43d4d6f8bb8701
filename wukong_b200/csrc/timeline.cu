// Host side of the decode-step timeline (diagnostic build libwukong_timeline.so,
// compiled with -DWK_TIMELINE; in the default library the first two entry
// points return -1).  No counterpart in the reference.
#include "timeline.cuh"
#include "wukong_internal.cuh"

namespace wk {
namespace {

#ifdef WK_TIMELINE
TimelineBuf g_tl;
#endif

// smallest step of %globaltimer seen by one thread (bounded loop)
__global__ void timer_step_kernel(unsigned long long *out) {
    uint64_t best = ~0ull, prev = globaltimer_ns();
    int changes = 0;
    for (int i = 0; i < (1 << 22) && changes < 64; ++i) {
        const uint64_t t = globaltimer_ns();
        if (t != prev) {
            if (t - prev < best) best = t - prev;
            prev = t;
            ++changes;
        }
    }
    *out = best;
}

}  // namespace
}  // namespace wk

using namespace wk;

extern "C" {

int wk_timeline_init(int slots, int blocks) {
#ifdef WK_TIMELINE
    ensure_init();
    if (slots <= 0 || blocks <= 0) return fail("timeline: slots %d, blocks %d", slots, blocks);
    if (!g_tl.stamps) {
        WK_CHECK(cudaMalloc(&g_tl.stamps, (size_t)slots * blocks * kTlStamps * 8));
        WK_CHECK(cudaMalloc(&g_tl.info, (size_t)slots * 4 * 4));
        WK_CHECK(cudaMalloc(&g_tl.count, 8));
        g_tl.done = g_tl.count + 1;
        g_tl.slots = slots;
        g_tl.blocks = blocks;
    } else if (slots != g_tl.slots || blocks != g_tl.blocks) {
        return fail("timeline: already initialised with %d slots, %d blocks", g_tl.slots, g_tl.blocks);
    }
    WK_CHECK(cudaMemsetAsync(g_tl.stamps, 0, (size_t)slots * blocks * kTlStamps * 8, stream()));
    WK_CHECK(cudaMemsetAsync(g_tl.info, 0, (size_t)slots * 4 * 4, stream()));
    WK_CHECK(cudaMemsetAsync(g_tl.count, 0, 8, stream()));
    WK_CHECK(cudaStreamSynchronize(stream()));
    timeline_bind_gemv(g_tl);
    timeline_bind_attn(g_tl);
    return 0;
#else
    (void)slots;
    (void)blocks;
    return fail("timeline: this is not the timeline build (python -m wukong_b200.build --timeline)");
#endif
}

// Copies the records to the host: info [slots][4] (kind, N, K, CTAs) and
// stamps [slots][blocks][9] (start, wait return, end, phases 0..5; ns).
// Returns the number of launches recorded (slot s holds launch s mod slots).
int wk_timeline_read(int *info, unsigned long long *stamps) {
#ifdef WK_TIMELINE
    if (!g_tl.stamps) return fail("timeline: not initialised");
    WK_CHECK(cudaStreamSynchronize(stream()));
    int count = 0;
    WK_CHECK(cudaMemcpy(&count, g_tl.count, 4, cudaMemcpyDeviceToHost));
    WK_CHECK(cudaMemcpy(info, g_tl.info, (size_t)g_tl.slots * 4 * 4, cudaMemcpyDeviceToHost));
    WK_CHECK(cudaMemcpy(stamps, g_tl.stamps, (size_t)g_tl.slots * g_tl.blocks * kTlStamps * 8,
                        cudaMemcpyDeviceToHost));
    return count;
#else
    (void)info;
    (void)stamps;
    return fail("timeline: this is not the timeline build");
#endif
}

// Smallest observed step of the %globaltimer clock in ns (the resolution of the
// stamps), or -1.
long long wk_timeline_resolution_ns(void) {
    ensure_init();
    unsigned long long *d = nullptr, h = 0;
    WK_CHECK(cudaMalloc(&d, 8));
    timer_step_kernel<<<1, 1, 0, stream()>>>(d);
    WK_CHECK(cudaGetLastError());
    WK_CHECK(cudaMemcpyAsync(&h, d, 8, cudaMemcpyDeviceToHost, stream()));
    WK_CHECK(cudaStreamSynchronize(stream()));
    WK_CHECK(cudaFree(d));
    return h == ~0ull ? -1 : (long long)h;
}

}  // extern "C"
