// Decode-step timeline: a diagnostic build (-DWK_TIMELINE, libwukong_timeline.so)
// in which every GEMV and decode-attention launch records, per CTA, %globaltimer
// at its start, after griddepcontrol.wait, at up to six phase marks and at its
// end.  Launches take slots in stream order: a launch reads the slot counter
// after its wait (the previous launch has completed by then) and its last CTA
// advances it.  In the default build Timeline is empty and compiles away.
#pragma once
#include "common.cuh"

namespace wk {

constexpr int kTlStamps = 9;  // start, wait return, end, phases 0..5

struct TimelineBuf {
    unsigned long long *stamps = nullptr;  // [slots][blocks][kTlStamps]
    int *info = nullptr;                   // [slots][4]: kind, N, K, CTAs
    int *count = nullptr;                  // next slot
    int *done = nullptr;                   // CTAs of the current launch that finished
    int slots = 0, blocks = 0;
};

#ifdef WK_TIMELINE
// one copy per translation unit, set by that unit's timeline_bind_* function
static __constant__ TimelineBuf c_tl;

struct Timeline {
    uint64_t t0, t1 = 0, ph[6] = {0, 0, 0, 0, 0, 0};
    int slot = -1;
    __device__ Timeline() : t0(globaltimer_ns()) {}
    // after griddepcontrol.wait: kind (the GEMV epilogue, 100.. for attention), shape
    __device__ void mark(int kind, int n, int k) {
        t1 = globaltimer_ns();
        if (threadIdx.x != 0 || !c_tl.stamps) return;
        slot = *(volatile int *)c_tl.count;
        if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0) {
            int *in = c_tl.info + (slot % c_tl.slots) * 4;
            in[0] = kind;
            in[1] = n;
            in[2] = k;
            in[3] = gridDim.x * gridDim.y * gridDim.z;
        }
    }
    __device__ void phase(int i) {
        if (threadIdx.x == 0 && ph[i] == 0) ph[i] = globaltimer_ns();
    }
    __device__ ~Timeline() {
        if (threadIdx.x != 0 || slot < 0) return;
        const uint64_t t2 = globaltimer_ns();
        const int b = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
        if (b < c_tl.blocks) {
            unsigned long long *p = c_tl.stamps + ((size_t)(slot % c_tl.slots) * c_tl.blocks + b) * kTlStamps;
            p[0] = t0;
            p[1] = t1;
            p[2] = t2;
            for (int i = 0; i < 6; ++i) p[3 + i] = ph[i];
        }
        __threadfence();
        if (atomicAdd(c_tl.done, 1) == (int)(gridDim.x * gridDim.y * gridDim.z) - 1) {
            *c_tl.done = 0;
            __threadfence();
            atomicExch(c_tl.count, slot + 1);
        }
    }
};
#else
struct Timeline {
    __device__ void mark(int, int, int) {}
    __device__ void phase(int) {}
};
#endif

// bind the buffers in gemv.cu / attention.cu (timeline build; no-ops otherwise)
void timeline_bind_gemv(const TimelineBuf &b);
void timeline_bind_attn(const TimelineBuf &b);

}  // namespace wk
