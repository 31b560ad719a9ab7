// Tensor-parallel exchanges over NVLink peer memory (one process per GPU).
//
// Each rank owns a receive buffer that every peer maps (CUDA IPC). A value a
// rank contributes travels as one 64-bit word {tag, payload} stored straight
// into every peer's buffer with a relaxed system-scope store (8-byte stores
// are single-copy atomic); a reader polls the words in its own buffer until
// the tag of the current exchange appears. There is no flag and no fence:
// the tag is the flag. One exchange is one small kernel, so a per-projection
// all-reduce costs one P2P store and one poll instead of a library
// collective's launch and protocol latency.
//
// Tags: every rank keeps a device generation counter; the exchanges of a
// token run in the same order on every rank, so exchange number g carries
// tag g + 1 everywhere. Buffers are double-buffered by g & 1: a rank cannot
// start exchange g + 2 before every peer has finished exchange g (finishing
// g + 1 needs every peer's g + 1 contribution, which a peer sends only after
// its exchange g kernel ended), so a region is never overwritten while a
// peer still reads it. Words are zero at creation (tag 0 never matches).
//
// Every poll is bounded (PollClock): a timeout reports kStatusWaitTimeout
// and the kernel finishes with what it has; nothing spins forever. Plain
// peer loads and stores only -- no multicast, no TMA on peer memory.

#include <cstring>

namespace h4b {

__device__ __forceinline__ void ll_store_sys(unsigned long long* p, unsigned long long w) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ll_load_sys(const unsigned long long* p) {
    unsigned long long w;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

// Word i of the slot that `src` fills in buffer `buf` for exchange parity `parity`.
__device__ __forceinline__ unsigned long long* tp_slot(const h4b_tp_group& g, unsigned long long* buf, int parity,
                                                       int src) {
    return buf + (static_cast<size_t>(parity) * g.world + src) * g.capacity;
}

// Sends payload words[0, n) of this rank to every rank (itself included).
__device__ __forceinline__ void tp_send(const h4b_tp_group& g, uint32_t tag, int parity, int i, uint32_t payload) {
    const unsigned long long w = (static_cast<unsigned long long>(tag) << 32) | payload;
    for (int p = 0; p < g.world; ++p) ll_store_sys(tp_slot(g, g.buffers[p], parity, g.rank) + i, w);
}

// Polls word i of `src`'s slot in this rank's buffer until it carries `tag`;
// returns the payload (0 after a timeout).
__device__ __forceinline__ uint32_t tp_receive(const h4b_tp_group& g, uint32_t tag, int parity, int src, int i) {
    const unsigned long long* p = tp_slot(g, g.buffers[g.rank], parity, src) + i;
    PollClock clock;
    for (;;) {
        const unsigned long long w = ll_load_sys(p);
        if (static_cast<uint32_t>(w >> 32) == tag) return static_cast<uint32_t>(w);
        if (poll_expired(clock)) return 0u;
    }
}

__device__ __forceinline__ void tp_finish(const h4b_tp_group& g, uint32_t gen) {
    __syncthreads();
    if (threadIdx.x == 0) *g.generation = gen + 1;
}

// value[0] <- max over ranks of value[0] (non-negative floats: the absmax
// a quantisation scale is made from; max is order-free).
__global__ void tp_allreduce_max_kernel(const h4b_tp_group g, float* value) {
    const uint32_t gen = *g.generation, tag = gen + 1;
    const int parity = gen & 1;
    if (threadIdx.x == 0) tp_send(g, tag, parity, 0, __float_as_uint(*value));
    float v = 0.f;  // lanes >= world keep 0, below any absmax
    if (threadIdx.x < g.world) v = __uint_as_float(tp_receive(g, tag, parity, threadIdx.x, 0));
    const float m = warp_max(v);  // all 32 lanes of the one warp
    if (threadIdx.x == 0) *value = m;
    tp_finish(g, gen);
}

// x[i] += float(sum over ranks of acc[i]) * dequant(absmax) * w_scale[i]:
// the K-split projection's int32 row sums added exactly across ranks, then
// the residual epilogue (decode.cu's residual_acc_kernel arithmetic).
__global__ void __launch_bounds__(1024) tp_allreduce_sum_residual_kernel(const h4b_tp_group g, const int32_t* acc,
                                                                          float* x, const float* absmax,
                                                                          const float* w_scale, int n) {
    const uint32_t gen = *g.generation, tag = gen + 1;
    const int parity = gen & 1;
    for (int i = threadIdx.x; i < n; i += blockDim.x) tp_send(g, tag, parity, i, static_cast<uint32_t>(acc[i]));
    const float scale = dequant_scale(*absmax);
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        int32_t total = 0;
        for (int src = 0; src < g.world; ++src) total += static_cast<int32_t>(tp_receive(g, tag, parity, src, i));
        x[i] = __fadd_rn(x[i], __fmul_rn(__fmul_rn(static_cast<float>(total), scale), w_scale[i]));
    }
    tp_finish(g, gen);
}

// Each rank's greedy candidate (its largest logit, global vocabulary index)
// to every rank: pairs[2 r] = value, pairs[2 r + 1] = index of rank r.
__global__ void tp_gather_best_kernel(const h4b_tp_group g, const float* logits, const int32_t* local_index,
                                      int vocab_offset, double* pairs) {
    const uint32_t gen = *g.generation, tag = gen + 1;
    const int parity = gen & 1;
    if (threadIdx.x == 0) {
        const int local = *local_index;
        tp_send(g, tag, parity, 0, __float_as_uint(logits[local]));
        tp_send(g, tag, parity, 1, static_cast<uint32_t>(local + vocab_offset));
    }
    if (threadIdx.x < g.world) {
        const int src = threadIdx.x;
        pairs[2 * src] = static_cast<double>(__uint_as_float(tp_receive(g, tag, parity, src, 0)));
        pairs[2 * src + 1] = static_cast<double>(static_cast<int32_t>(tp_receive(g, tag, parity, src, 1)));
    }
    tp_finish(g, gen);
}

int validate_tp_group(const h4b_tp_group* g, int words) {
    if (!g || g->world < 1 || g->world > H4B_TP_MAX_RANKS || g->rank < 0 || g->rank >= g->world || !g->generation)
        return H4B_EINVAL;
    if (words > g->capacity) return H4B_EINVAL;
    for (int r = 0; r < g->world; ++r)
        if (!g->buffers[r] || (reinterpret_cast<uintptr_t>(g->buffers[r]) & 7)) return H4B_EINVAL;
    return 0;
}

}  // namespace h4b

extern "C" long long h4b_tp_buffer_bytes(int world, int capacity) {
    if (world < 1 || world > H4B_TP_MAX_RANKS || capacity < 2) return H4B_EINVAL;
    return 2ll * world * capacity * static_cast<long long>(sizeof(unsigned long long));
}

extern "C" int h4b_ipc_alloc(long long bytes, void** ptr, void* handle) {
    if (bytes <= 0 || !ptr || !handle) return H4B_EINVAL;
    H4B_CUDA_TRY(cudaMalloc(ptr, static_cast<size_t>(bytes)));
    cudaError_t e = cudaMemset(*ptr, 0, static_cast<size_t>(bytes));
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), *ptr);
    if (e != cudaSuccess) {
        cudaFree(*ptr);
        *ptr = nullptr;
        return static_cast<int>(e);
    }
    return 0;
}

extern "C" int h4b_ipc_open(const void* handle, void** ptr) {
    if (!handle || !ptr) return H4B_EINVAL;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    H4B_CUDA_TRY(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
    return 0;
}

extern "C" int h4b_ipc_close(void* ptr) {
    H4B_CUDA_TRY(cudaIpcCloseMemHandle(ptr));
    return 0;
}

extern "C" int h4b_ipc_free(void* ptr) {
    H4B_CUDA_TRY(cudaFree(ptr));
    return 0;
}

extern "C" int h4b_tp_allreduce_max(const h4b_tp_group* group, float* value, void* stream) {
    int rc = h4b::validate_tp_group(group, 1);
    if (rc) return rc;
    if (!value) return H4B_EINVAL;
    h4b::tp_allreduce_max_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(*group, value);
    H4B_CUDA_TRY(cudaGetLastError());
    return 0;
}

extern "C" int h4b_tp_allreduce_sum_residual(const h4b_tp_group* group, const int32_t* acc, float* x,
                                             const float* absmax, const float* w_scales, int n, void* stream) {
    int rc = h4b::validate_tp_group(group, n);
    if (rc) return rc;
    if (!acc || !x || !absmax || !w_scales || n < 1) return H4B_EINVAL;
    h4b::tp_allreduce_sum_residual_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(*group, acc, x, absmax,
                                                                                           w_scales, n);
    H4B_CUDA_TRY(cudaGetLastError());
    return 0;
}

extern "C" int h4b_tp_gather_best(const h4b_tp_group* group, const float* logits, const int32_t* local_index,
                                  int vocab_offset, double* pairs, void* stream) {
    int rc = h4b::validate_tp_group(group, 2);
    if (rc) return rc;
    if (!logits || !local_index || !pairs) return H4B_EINVAL;
    h4b::tp_gather_best_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(*group, logits, local_index,
                                                                               vocab_offset, pairs);
    H4B_CUDA_TRY(cudaGetLastError());
    return 0;
}
