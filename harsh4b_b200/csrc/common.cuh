// Shared device helpers for the sm_100a decode kernels: status reporting,
// mbarrier + bulk-copy (TMA engine) primitives, programmatic dependent
// launch, and block reductions.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <atomic>
#include <mutex>

#include "../../include/harsh4b_b200.h"

namespace h4b {

// ---- status ------------------------------------------------------------
// Kernels never trap. A bounded wait that gives up ORs a code into this
// word; h4b_get_status() reads and clears it from the host. (The library is
// one translation unit, harsh4b_b200.cu, so this is its only definition.)
__device__ int g_status = 0;

constexpr int kMaxDevices = 64;  // per-device host-side state is kept for device ordinals below this

constexpr int kStatusWaitTimeout = 1;     // an mbarrier wait ran out of time
constexpr int kStatusBadToken = 2;        // token id outside the vocabulary
constexpr int kStatusBadPosition = 4;     // decode position beyond capacity

__device__ __forceinline__ void report(int code) { atomicOr(&g_status, code); }

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// A wait gives up after this long; normal waits last microseconds.
constexpr uint64_t kWaitLimitNs = 1000000000ull;

// True once any kernel has given up on a wait: later kernels then skip their
// work, so a failure costs one wait limit instead of one per launch.
__device__ __forceinline__ bool wait_failed_before() {
    return (*reinterpret_cast<volatile int*>(&g_status) & kStatusWaitTimeout) != 0;
}

// ---- optional phase timeline ----------------------------------------------
// Built with -DH4B_PHASE_TRACE, H4B_TRACE(ev) records %globaltimer for event
// `ev` (< 2048) on three CTAs (first, middle, last) into g_phase_trace, which
// h4b_phase_trace copies out. In the normal build it compiles to nothing.
#ifdef H4B_PHASE_TRACE
__device__ unsigned long long g_phase_trace[3][2048];
__device__ __forceinline__ int trace_slot() {
    const unsigned c = blockIdx.x;
    return c == 0 ? 0 : (c == gridDim.x / 2 ? 1 : (c == gridDim.x - 1 ? 2 : -1));
}
#define H4B_TRACE_ANY(ev)                                                             \
    do {                                                                              \
        const int _s = ::h4b::trace_slot();                                           \
        if (_s >= 0) ::h4b::g_phase_trace[_s][(ev)] = ::h4b::globaltimer_ns();        \
    } while (0)
#define H4B_TRACE(ev)                                \
    do {                                             \
        if (threadIdx.x == 0) H4B_TRACE_ANY(ev);     \
    } while (0)
// Per-CTA timestamps (all CTAs): g_phase_all[cta][ev], ev < 32.
__device__ unsigned long long g_phase_all[1024][32];
#define H4B_TRACE_CTA(ev)                                                                    \
    do {                                                                                     \
        if (threadIdx.x == 0) ::h4b::g_phase_all[blockIdx.x][(ev)] = ::h4b::globaltimer_ns(); \
    } while (0)
#define H4B_TRACE_VAL(ev, val)                                                           \
    do {                                                                                 \
        const int _s = ::h4b::trace_slot();                                              \
        if (_s >= 0) ::h4b::g_phase_trace[_s][(ev)] = static_cast<unsigned long long>(val); \
    } while (0)
#else
#define H4B_TRACE_CTA(ev) do { } while (0)
#define H4B_TRACE_VAL(ev, val) do { } while (0)
#define H4B_TRACE_ANY(ev) do { } while (0)
#define H4B_TRACE(ev) do { } while (0)
#endif

// ---- programmatic dependent launch ---------------------------------------
// Everything before pdl_wait() may only touch data no earlier kernel in the
// stream writes (weights, scales, tables). pdl_trigger() lets the next
// kernel's CTAs start their own weight prefetch.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---- mbarrier ---------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}"
                 :: "r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}"
                 :: "r"(smem_addr(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(done) : "r"(smem_addr(bar)), "r"(parity) : "memory");
    return done != 0;
}

// try_wait that may park the thread for up to `hint_ns` inside the
// instruction; it returns as soon as the phase completes.
__device__ __forceinline__ bool mbar_try_wait_hint(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t done;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(done) : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns) : "memory");
    return done != 0;
}

// Bounded wait for the phase with the given parity to complete. Returns
// false (and reports) when the time limit passes. The waiting thread parks
// inside try_wait rather than spinning, so idle waiters take no issue slots
// from the warps doing work; the clock is read only between parkings.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns = kWaitLimitNs) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t start = globaltimer_ns();
    while (!mbar_try_wait_hint(bar, parity, 20000)) {
        if (globaltimer_ns() - start > limit_ns) {
            report(kStatusWaitTimeout);
            return false;
        }
    }
    return true;
}

// 1-D bulk copy global -> shared through the TMA engine, completing on the
// mbarrier's transaction count. dst, src and bytes must be 16-byte multiples.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar)) : "memory");
}

// 4-byte asynchronous global -> shared copy (no register round trip).
__device__ __forceinline__ void async_copy4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" :: "r"(smem_addr(dst)), "l"(src) : "memory");
}
// 16-byte asynchronous copy through L2 only (data another SM may have
// written in an earlier launch); both addresses 16-byte aligned.
__device__ __forceinline__ void async_copy16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(smem_addr(dst)), "l"(src) : "memory");
}
// Closes the async copies issued so far into one group.
__device__ __forceinline__ void async_copy_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// Waits until at most N of this thread's committed copy groups are pending.
template <int N>
__device__ __forceinline__ void async_copy_wait_prior() {
    asm volatile("cp.async.wait_group %0;" :: "n"(N) : "memory");
}
__device__ __forceinline__ void async_copy_wait_all() {
    asm volatile("cp.async.wait_all;" ::: "memory");
}

// ---- tagged exchange words ------------------------------------------------------
// A 64-bit word carries a 32-bit payload (low half) and a 32-bit tag (high
// half) and is written and read with single 8-byte accesses, which are
// single-copy atomic: a reader that sees the tag it expects also sees the
// payload stored with it. Producers store with no fence and consumers poll
// the words themselves, so a cross-SM handoff costs one store plus one load
// instead of store, fence, flag, poll and load.
__device__ __forceinline__ unsigned long long ll_pack(float v, uint32_t tag) {
    return (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(v);
}
__device__ __forceinline__ uint32_t ll_tag(unsigned long long w) { return static_cast<uint32_t>(w >> 32); }
__device__ __forceinline__ float ll_value(unsigned long long w) {
    return __uint_as_float(static_cast<uint32_t>(w & 0xFFFFFFFFull));
}
__device__ __forceinline__ void ll_store(unsigned long long* p, float v, uint32_t tag) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" :: "l"(p), "l"(ll_pack(v, tag)) : "memory");
}
__device__ __forceinline__ void ll_store_raw2(unsigned long long* p, unsigned long long a, unsigned long long b) {
    asm volatile("st.relaxed.gpu.global.v2.u64 [%0], {%1, %2};" :: "l"(p), "l"(a), "l"(b) : "memory");
}
// Two adjacent words (p 16-byte aligned).
__device__ __forceinline__ void ll_store2(unsigned long long* p, float a, float b, uint32_t tag) {
    ll_store_raw2(p, ll_pack(a, tag), ll_pack(b, tag));
}
__device__ __forceinline__ ulonglong2 ll_load2(const unsigned long long* p) {
    ulonglong2 w;
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(w.x), "=l"(w.y) : "l"(p) : "memory");
    return w;
}
__device__ __forceinline__ unsigned long long ll_load(const unsigned long long* p) {
    unsigned long long w;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

// Bounded polling: a poll loop calls poll_expired() between rounds; it
// returns true (after reporting) once the wait limit has passed or another
// wait has already failed. Rounds follow each other without a sleep: a round
// is already one L2 round trip, and a 96 ns back-off between rounds measured
// 1 % slower on the persistent decode (later detection of each handoff).
struct PollClock {
    uint64_t start = 0;
    uint32_t rounds = 0;
};
__device__ __forceinline__ bool poll_expired(PollClock& c) {
    if (c.rounds++ == 0) {
        c.start = globaltimer_ns();
        return false;
    }
    if ((c.rounds & 255) != 0) return false;
    if (wait_failed_before()) return true;
    if (globaltimer_ns() - c.start > kWaitLimitNs) {
        report(kStatusWaitTimeout);
        return true;
    }
    return false;
}

// ---- grid-scope release / acquire counters ------------------------------------
// Release-add: every write this thread has observed (the CTA's writes, after
// a CTA barrier) is visible at GPU scope before the count moves.
__device__ __forceinline__ void red_release_add(uint32_t* counter, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" :: "l"(counter), "r"(v) : "memory");
}
// Acquire-release add that returns the previous count (last-arriver tests).
__device__ __forceinline__ uint32_t atom_acq_rel_add(uint32_t* counter, uint32_t v) {
    uint32_t prev;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(prev) : "l"(counter), "r"(v) : "memory");
    return prev;
}

// ---- named barrier among a subset of warps ------------------------------------
__device__ __forceinline__ void named_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(threads) : "memory");
}

// ---- reductions -------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Sum over `warps` warps (threads 0 .. 32*warps-1) synchronised with named
// barrier `bar`; every participating thread gets the total. `scratch` holds
// at least 32 floats. The order is fixed, so the result is deterministic.
__device__ __forceinline__ float group_sum(float v, float* scratch, int warps, int bar) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    if (lane == 0) scratch[warp] = v;
    named_sync(bar, warps * 32);
    float total = 0.f;
    for (int w = 0; w < warps; ++w) total += scratch[w];
    named_sync(bar, warps * 32);
    return total;
}

__device__ __forceinline__ float group_max(float v, float* scratch, int warps, int bar) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_max(v);
    if (lane == 0) scratch[warp] = v;
    named_sync(bar, warps * 32);
    float total = scratch[0];
    for (int w = 1; w < warps; ++w) total = fmaxf(total, scratch[w]);
    named_sync(bar, warps * 32);
    return total;
}

// group_max without the closing barrier: `scratch` must not be written
// again before the caller's next barrier on `bar`.
__device__ __forceinline__ float group_max_open(float v, float* scratch, int warps, int bar) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_max(v);
    if (lane == 0) scratch[warp] = v;
    named_sync(bar, warps * 32);
    float total = scratch[0];
    for (int w = 1; w < warps; ++w) total = fmaxf(total, scratch[w]);
    return total;
}

// Non-negative floats order like their bit patterns, so an unsigned
// atomicMax on the bits is an exact, order-independent float max.
__device__ __forceinline__ void atomic_max_nonneg(float* slot, float value) {
    atomicMax(reinterpret_cast<unsigned int*>(slot), __float_as_uint(value));
}

// Per-token absmax int8 quantisation contract (shared with the oracle):
//   m = max(absmax, 1e-5); qs = 127 / m; q = clamp(rint(v * qs), -127, 127);
//   dequant scale = m / 127.
__device__ __forceinline__ float quant_multiplier(float absmax) {
    return __fdiv_rn(127.0f, fmaxf(absmax, 1e-5f));
}
__device__ __forceinline__ float dequant_scale(float absmax) {
    return __fdiv_rn(fmaxf(absmax, 1e-5f), 127.0f);
}
__device__ __forceinline__ int quantize_one(float v, float qs) {
    int q = __float2int_rn(__fmul_rn(v, qs));
    return max(-127, min(127, q));
}

// exp(x) by Cody-Waite range reduction (x = n ln2 + r, |r| <= ln2/2, with
// ln2 split into a short high part and a low correction) and the degree-7
// Taylor polynomial of exp(r) in Horner form, scaled exactly by 2^n. Inputs
// below -87 give 0; inputs above 88 are clamped. One IEEE op per step, so
// a CPU implementation with the same steps returns the same bits (the test
// oracle does); within 2 ulp of exp on [-87, 88].
__device__ __forceinline__ float exp_cw(float x) {
    if (x < -87.0f) return 0.0f;
    x = fminf(x, 88.0f);
    const float n = rintf(__fmul_rn(x, 1.44269504f));
    float r = __fmaf_rn(n, -0.693145751953125f, x);
    r = __fmaf_rn(n, -1.42860682e-06f, r);
    float p = 1.98412698e-04f;
    p = __fmaf_rn(p, r, 1.38888889e-03f);
    p = __fmaf_rn(p, r, 8.33333333e-03f);
    p = __fmaf_rn(p, r, 4.16666667e-02f);
    p = __fmaf_rn(p, r, 1.66666667e-01f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    return __fmul_rn(p, __int_as_float((static_cast<int>(n) + 127) << 23));
}

// SiLU(gate) * up in the order every SwiGLU of this library uses.
__device__ __forceinline__ float swiglu_one(float g, float u) {
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, exp_cw(-g))), u);
}

// Argmax key: larger value wins, ties go to the smaller index (numpy's
// first-occurrence rule). Values are mapped to an order-preserving uint.
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t index) {
    uint32_t b = __float_as_uint(v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return (static_cast<unsigned long long>(b) << 32) | (0xFFFFFFFFu - index);
}

}  // namespace h4b

#define H4B_CUDA_TRY(expr)                                   \
    do {                                                     \
        cudaError_t _e = (expr);                             \
        if (_e != cudaSuccess) return static_cast<int>(_e);  \
    } while (0)
