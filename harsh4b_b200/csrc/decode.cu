// Decode-step orchestration and the small operator kernels.
//
// One token (cpu_lightspark.py:424-468) is a chain of 5 * layers + 3 kernel
// launches on one stream, each launched with programmatic stream
// serialisation so a kernel's weight prefetch overlaps its predecessor:
//
//   embed(+reset) -> per layer { qkv GEMV [RMSNorm+quant prologue]
//                               -> attention [qk-norm, RoPE, KV append, split-K, merge, absmax]
//                               -> o GEMV [quant prologue, residual epilogue]
//                               -> gate/up GEMV [RMSNorm+quant prologue, SwiGLU+absmax epilogue]
//                               -> down GEMV [quant prologue, residual epilogue] }
//   -> LM head GEMV [RMSNorm+quant prologue, logits+argmax epilogue] -> finalize
//
// The token id and position live in device memory, so one captured CUDA
// graph serves every step of a session.
#include <algorithm>
#include <new>

#include "common.cuh"

namespace h4b {

__global__ void __launch_bounds__(256) embed_kernel(const int32_t* token, const uint8_t* embedding,
                                                     const float* scales, float* out, int vocab, int hidden,
                                                     const int32_t* position, int capacity, float* absmax,
                                                     int absmax_n, unsigned long long* argmax_key) {
    pdl_wait();
    pdl_trigger();
    const int t = *token;
    const bool ok = t >= 0 && t < vocab;
    if (threadIdx.x == 0) {
        if (!ok) report(kStatusBadToken);
        if (position && *position >= capacity) report(kStatusBadPosition);
        if (argmax_key) *argmax_key = 0ull;
    }
    for (int i = threadIdx.x; i < absmax_n; i += blockDim.x) absmax[i] = 0.f;
    // cpu_lightspark.py:341-349: low nibble -> even column, times the row scale.
    const float scale = ok ? scales[t] : 0.f;
    const uint8_t* row = embedding + static_cast<size_t>(ok ? t : 0) * (hidden >> 1);
    for (int j = threadIdx.x; j < (hidden >> 1); j += blockDim.x) {
        const int8_t byte = static_cast<int8_t>(row[j]);
        const int lo = static_cast<int8_t>(byte << 4) >> 4;
        const int hi = byte >> 4;
        out[2 * j] = ok ? __fmul_rn(static_cast<float>(lo), scale) : 0.f;
        out[2 * j + 1] = ok ? __fmul_rn(static_cast<float>(hi), scale) : 0.f;
    }
}

__global__ void finalize_kernel(const unsigned long long* argmax_key, int32_t* next_token, int32_t* token,
                                int32_t* position) {
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x == 0) {
        const int32_t id = static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(*argmax_key & 0xFFFFFFFFull));
        *next_token = id;
        if (token) *token = id;
        *position += 1;
    }
}

// Same arithmetic and reduction order as the GEMV RMSNorm prologue
// (256 threads, groups of 8 columns, fmaf accumulation, fixed warp order).
__global__ void __launch_bounds__(256) rmsnorm_kernel(const float* x, const float* w, float* out, int n, float eps) {
    __shared__ float red[32];
    const int groups = n >> 3;
    float ss = 0.f;
    for (int g = threadIdx.x; g < groups; g += 256) {
        const float4 a = *reinterpret_cast<const float4*>(x + 8 * g);
        const float4 b = *reinterpret_cast<const float4*>(x + 8 * g + 4);
        const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = __fmaf_rn(v[e], v[e], ss);
    }
    ss = group_sum(ss, red, 8, 1);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(n)), eps)));
    for (int i = threadIdx.x; i < n; i += 256) out[i] = __fmul_rn(__fmul_rn(x[i], inv), w[i]);
}

__global__ void __launch_bounds__(256) quantize_kernel(const float* v, int8_t* q, float* scale_out, int n) {
    __shared__ float red[32];
    float local = 0.f;
    for (int i = threadIdx.x; i < n; i += 256) local = fmaxf(local, fabsf(v[i]));
    const float m = group_max(local, red, 8, 1);
    const float qs = quant_multiplier(m);
    for (int i = threadIdx.x; i < n; i += 256) q[i] = static_cast<int8_t>(quantize_one(v[i], qs));
    if (threadIdx.x == 0) *scale_out = dequant_scale(m);
}

// x[r] += float(acc[r]) * dequant_scale(*absmax) * w_scale[r]: the residual
// epilogue applied to int32 row sums reduced across a tensor-parallel group.
__global__ void residual_acc_kernel(float* x, const int32_t* acc, const float* absmax, const float* w_scale, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float v = __fmul_rn(__fmul_rn(static_cast<float>(acc[i]), dequant_scale(*absmax)), w_scale[i]);
    x[i] = __fadd_rn(x[i], v);
}

__global__ void add_kernel(float* x, const float* y, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[i] = __fadd_rn(x[i], y[i]);
}

__global__ void __launch_bounds__(1024) argmax_kernel(const float* v, int n, int32_t* out) {
    __shared__ unsigned long long keys[32];
    unsigned long long best = 0ull;
    for (int i = threadIdx.x; i < n; i += 1024) {
        const unsigned long long k = argmax_key(v[i], static_cast<uint32_t>(i));
        best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
    }
    if ((threadIdx.x & 31) == 0) keys[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 0; w < 32; ++w) best = keys[w] > best ? keys[w] : best;
        *out = static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(best & 0xFFFFFFFFull));
    }
}

template <typename K, typename... Args>
static int launch_pdl(K kernel, dim3 grid, dim3 block, cudaStream_t stream, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    H4B_CUDA_TRY(cudaLaunchKernelEx(&cfg, kernel, args...));
    return 0;
}

static size_t kv_elem_bytes(int kv_dtype) { return kv_dtype == 0 ? 4 : 2; }

int validate(const h4b_model* m, const h4b_state* s) {
    if (!m || !s) return H4B_EINVAL;
    if (m->head_dim != kHeadDim) return H4B_EUNSUPPORTED;
    if (m->layers < 1 || m->kv_heads < 1 || m->heads % m->kv_heads) return H4B_EINVAL;
    const int groups = m->heads / m->kv_heads;
    if (groups > 8) return H4B_EUNSUPPORTED;
    if ((m->hidden & 31) || (m->intermediate & 31) || (m->heads * m->head_dim) & 31) return H4B_EUNSUPPORTED;
    if (m->intermediate % kSwigluBlock) return H4B_EUNSUPPORTED;
    if (s->capacity < 1 || s->capacity > m->max_pos) return H4B_EINVAL;
    if (s->kv_dtype != 0 && s->kv_dtype != 1) return H4B_EINVAL;
    if (s->attn_splits < 1 || s->attn_splits > 64) return H4B_EINVAL;
    const void* required[] = {m->w_qkv, m->s_qkv, m->w_o, m->s_o, m->w_gate_up, m->s_gate_up, m->w_down,
                              m->s_down, m->w_embed, m->s_embed, m->norm_in, m->norm_post, m->norm_q, m->norm_k,
                              m->norm_final, m->rope_cos, m->rope_sin, s->k_cache, s->v_cache, s->position,
                              s->token, s->next_token, s->x, s->qkv, s->attended, s->act, s->logits, s->absmax,
                              s->argmax_key};
    for (const void* p : required)
        if (!p || (reinterpret_cast<uintptr_t>(p) & 15)) return H4B_EINVAL;
    if (s->attn_splits > 1 && (!s->attn_partials || !s->attn_counters)) return H4B_EINVAL;
    return 0;
}

// Stages of one decode token; layer-indexed stages take `layer`.
enum Stage { STAGE_EMBED = 0, STAGE_QKV, STAGE_ATTN, STAGE_O, STAGE_GATE_UP, STAGE_DOWN, STAGE_LM_HEAD,
             STAGE_FINALIZE, STAGE_COUNT };

int launch_stage(const h4b_model* m, const h4b_state* s, int stage, int l, cudaStream_t stream, bool pdl) {
    const int H = m->hidden, I = m->intermediate, d = m->head_dim;
    const int q_size = m->heads * d, kv_size = m->kv_heads * d;
    const int qkv_rows = q_size + 2 * kv_size;
    const size_t kv_layer = static_cast<size_t>(m->kv_heads) * s->capacity * d * kv_elem_bytes(s->kv_dtype);
    if (l < 0 || l >= m->layers) return H4B_EINVAL;
    GemvArgs g = {};
    switch (stage) {
        case STAGE_EMBED:
            return launch_pdl(embed_kernel, dim3(1), dim3(256), stream, pdl, (const int32_t*)s->token, m->w_embed,
                              m->s_embed, s->x, m->vocab, H, (const int32_t*)s->position, s->capacity, s->absmax,
                              2 * m->layers, s->argmax_key);
        case STAGE_QKV:
            g.w = m->w_qkv + static_cast<size_t>(l) * qkv_rows * (H / 2);
            g.wscale = m->s_qkv + static_cast<size_t>(l) * qkv_rows;
            g.rows = qkv_rows; g.width = H;
            g.xin = s->x; g.gamma = m->norm_in + static_cast<size_t>(l) * H; g.eps = m->eps;
            g.out = s->qkv;
            return launch_gemv(PRO_RMSNORM, EPI_STORE, g, stream, pdl);
        case STAGE_ATTN: {
            AttnArgs a = {};
            a.q = s->qkv; a.knew = s->qkv + q_size; a.vnew = s->qkv + q_size + kv_size;
            a.q_norm = m->norm_q + static_cast<size_t>(l) * d;
            a.k_norm = m->norm_k + static_cast<size_t>(l) * d;
            a.rope_cos = m->rope_cos; a.rope_sin = m->rope_sin; a.eps = m->eps;
            a.kcache = static_cast<char*>(s->k_cache) + l * kv_layer;
            a.vcache = static_cast<char*>(s->v_cache) + l * kv_layer;
            a.head_stride = static_cast<long long>(s->capacity) * d;
            a.time_stride = d;
            a.position = s->position; a.capacity = s->capacity;
            a.groups = m->heads / m->kv_heads; a.kv_heads = m->kv_heads; a.splits = s->attn_splits;
            a.partials = s->attn_partials; a.counters = s->attn_counters;
            a.out = s->attended; a.absmax_out = s->absmax + 2 * l;
            return launch_attention(a, s->kv_dtype, 1, stream, pdl);
        }
        case STAGE_O:
            g.w = m->w_o + static_cast<size_t>(l) * H * (q_size / 2);
            g.wscale = m->s_o + static_cast<size_t>(l) * H;
            g.rows = H; g.width = q_size;
            g.xin = s->attended; g.absmax_in = s->absmax + 2 * l; g.out = s->x;
            return launch_gemv(PRO_QUANT_ABSMAX, EPI_RESIDUAL, g, stream, pdl);
        case STAGE_GATE_UP:
            g.w = m->w_gate_up + static_cast<size_t>(l) * 2 * I * (H / 2);
            g.wscale = m->s_gate_up + static_cast<size_t>(l) * 2 * I;
            g.rows = 2 * I; g.width = H;
            g.xin = s->x; g.gamma = m->norm_post + static_cast<size_t>(l) * H; g.eps = m->eps;
            g.out = s->act; g.absmax_out = s->absmax + 2 * l + 1;
            return launch_gemv(PRO_RMSNORM, EPI_SWIGLU, g, stream, pdl);
        case STAGE_DOWN:
            g.w = m->w_down + static_cast<size_t>(l) * H * (I / 2);
            g.wscale = m->s_down + static_cast<size_t>(l) * H;
            g.rows = H; g.width = I;
            g.xin = s->act; g.absmax_in = s->absmax + 2 * l + 1; g.out = s->x;
            return launch_gemv(PRO_QUANT_ABSMAX, EPI_RESIDUAL, g, stream, pdl);
        case STAGE_LM_HEAD:
            g.w = m->w_embed; g.wscale = m->s_embed; g.rows = m->vocab; g.width = H;
            g.xin = s->x; g.gamma = m->norm_final; g.eps = m->eps;
            g.out = s->logits; g.argmax_out = s->argmax_key;
            return launch_gemv(PRO_RMSNORM, EPI_ARGMAX, g, stream, pdl);
        case STAGE_FINALIZE:
            return launch_pdl(finalize_kernel, dim3(1), dim3(32), stream, pdl,
                              (const unsigned long long*)s->argmax_key, s->next_token, s->token, s->position);
        default:
            return H4B_EINVAL;
    }
}

int decode_step(const h4b_model* m, const h4b_state* s, cudaStream_t stream) {
    int r = validate(m, s);
    if (r) return r;
    if ((r = launch_stage(m, s, STAGE_EMBED, 0, stream, true))) return r;
    for (int l = 0; l < m->layers; ++l)
        for (int stage = STAGE_QKV; stage <= STAGE_DOWN; ++stage)
            if ((r = launch_stage(m, s, stage, l, stream, true))) return r;
    if ((r = launch_stage(m, s, STAGE_LM_HEAD, 0, stream, true))) return r;
    return launch_stage(m, s, STAGE_FINALIZE, 0, stream, true);
}

int prepare_persistent();  // persistent.cu
int prepare_sampling();    // sample.cu

int prepare_other_kernels() {
    int r = 0;
    if ((r = prepare_persistent())) return r;
    if ((r = prepare_sampling())) return r;
    if ((r = cudaFuncSetAttribute(gqa_split_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  subtile_smem_bytes<float>())))
        return r;
    if ((r = set_carveout(gqa_split_kernel<float>)) || (r = set_carveout(gqa_split_kernel<__half>)) ||
        (r = set_carveout(gqa_merge_kernel)) || (r = set_carveout(embed_kernel)) ||
        (r = set_carveout(finalize_kernel)))
        return r;
    return 0;
}

struct GraphHandle {
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
};

}  // namespace h4b

// ---------------------------------------------------------------------------
// C ABI

extern "C" int h4b_get_status(int* host_status) {
    if (!host_status) return H4B_EINVAL;
    H4B_CUDA_TRY(cudaDeviceSynchronize());
    H4B_CUDA_TRY(cudaMemcpyFromSymbol(host_status, h4b::g_status, sizeof(int)));
    const int zero = 0;
    H4B_CUDA_TRY(cudaMemcpyToSymbol(h4b::g_status, &zero, sizeof(int)));
    return 0;
}

extern "C" int h4b_device_info(int* sm, int* major, int* minor) {
    int dev = 0;
    H4B_CUDA_TRY(cudaGetDevice(&dev));
    if (sm) H4B_CUDA_TRY(cudaDeviceGetAttribute(sm, cudaDevAttrMultiProcessorCount, dev));
    if (major) H4B_CUDA_TRY(cudaDeviceGetAttribute(major, cudaDevAttrComputeCapabilityMajor, dev));
    if (minor) H4B_CUDA_TRY(cudaDeviceGetAttribute(minor, cudaDevAttrComputeCapabilityMinor, dev));
    return 0;
}

extern "C" int h4b_quantize_activation(const float* values, int8_t* quantized, float* scale_out, int n,
                                       void* stream) {
    if (!values || !quantized || !scale_out || n < 1) return H4B_EINVAL;
    h4b::quantize_kernel<<<1, 256, 0, static_cast<cudaStream_t>(stream)>>>(values, quantized, scale_out, n);
    return static_cast<int>(cudaGetLastError());
}

extern "C" int h4b_rmsnorm(const float* x, const float* weight, float* out, int n, float eps, void* stream) {
    if (!x || !weight || !out || n < 8 || (n & 7)) return H4B_EINVAL;
    if ((reinterpret_cast<uintptr_t>(x) & 15)) return H4B_EINVAL;
    h4b::rmsnorm_kernel<<<1, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, weight, out, n, eps);
    return static_cast<int>(cudaGetLastError());
}

extern "C" int h4b_add_inplace(float* x, const float* y, int n, void* stream) {
    if (!x || !y || n < 1) return H4B_EINVAL;
    h4b::add_kernel<<<(n + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, y, n);
    return static_cast<int>(cudaGetLastError());
}

extern "C" int h4b_embedding(const int32_t* token, const uint8_t* embedding, const float* scales, float* out,
                             int vocab, int hidden, void* stream) {
    if (!token || !embedding || !scales || !out || vocab < 1 || hidden < 2 || (hidden & 1)) return H4B_EINVAL;
    return h4b::launch_pdl(h4b::embed_kernel, dim3(1), dim3(256), static_cast<cudaStream_t>(stream), false, token,
                           embedding, scales, out, vocab, hidden, (const int32_t*)nullptr, 0, (float*)nullptr, 0,
                           (unsigned long long*)nullptr);
}

extern "C" int h4b_argmax(const float* logits, int n, int32_t* token_out, void* stream) {
    if (!logits || !token_out || n < 1) return H4B_EINVAL;
    h4b::argmax_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(logits, n, token_out);
    return static_cast<int>(cudaGetLastError());
}

extern "C" int h4b_validate(const h4b_model* model, const h4b_state* state) {
    return h4b::validate(model, state);
}

extern "C" int h4b_decode_stage(const h4b_model* model, const h4b_state* state, int stage, int layer,
                                void* stream) {
    const int rc = h4b::validate(model, state);
    if (rc) return rc;
    return h4b::launch_stage(model, state, stage, layer, static_cast<cudaStream_t>(stream), false);
}

extern "C" int h4b_prepare(void) {
    return h4b::prepare_kernels();
}

extern "C" int h4b_decode_step(const h4b_model* model, const h4b_state* state, void* stream) {
    return h4b::decode_step(model, state, static_cast<cudaStream_t>(stream));
}

namespace h4b {
int decode_persistent(const h4b_model* m, const h4b_state* s, cudaStream_t stream);  // persistent.cu

static int capture_step(const h4b_model* model, const h4b_state* state, void* stream, void** graph_out,
                        int (*step)(const h4b_model*, const h4b_state*, cudaStream_t)) {
    if (!graph_out) return H4B_EINVAL;
    int rc = validate(model, state);
    if (rc) return rc;
    if ((rc = prepare_kernels())) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    GraphHandle* h = new (std::nothrow) GraphHandle();
    if (!h) return H4B_EINVAL;
    cudaError_t e = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) { delete h; return static_cast<int>(e); }
    rc = step(model, state, s);
    e = cudaStreamEndCapture(s, &h->graph);
    if (rc || e != cudaSuccess) {
        if (h->graph) cudaGraphDestroy(h->graph);
        delete h;
        return rc ? rc : static_cast<int>(e);
    }
    e = cudaGraphInstantiate(&h->exec, h->graph, 0);
    if (e != cudaSuccess) {
        cudaGraphDestroy(h->graph);
        delete h;
        return static_cast<int>(e);
    }
    *graph_out = h;
    return 0;
}
}  // namespace h4b

extern "C" int h4b_graph_create(const h4b_model* model, const h4b_state* state, void* stream, void** graph_out) {
    return h4b::capture_step(model, state, stream, graph_out, h4b::decode_step);
}

extern "C" int h4b_graph_create_persistent(const h4b_model* model, const h4b_state* state, void* stream,
                                           void** graph_out) {
    return h4b::capture_step(model, state, stream, graph_out, h4b::decode_persistent);
}

extern "C" int h4b_graph_launch(void* graph, void* stream) {
    if (!graph) return H4B_EINVAL;
    return static_cast<int>(cudaGraphLaunch(static_cast<h4b::GraphHandle*>(graph)->exec,
                                            static_cast<cudaStream_t>(stream)));
}

extern "C" int h4b_graph_token(void* graph, const int32_t* token_host, int32_t* token_dev, const int32_t* next_dev,
                               int32_t* next_host, void* stream) {
    if (!graph || !token_host || !token_dev || !next_dev || !next_host) return H4B_EINVAL;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    H4B_CUDA_TRY(cudaMemcpyAsync(token_dev, token_host, sizeof(int32_t), cudaMemcpyHostToDevice, s));
    H4B_CUDA_TRY(cudaGraphLaunch(static_cast<h4b::GraphHandle*>(graph)->exec, s));
    H4B_CUDA_TRY(cudaMemcpyAsync(next_host, next_dev, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
    H4B_CUDA_TRY(cudaStreamSynchronize(s));
    return 0;
}

extern "C" int h4b_graph_destroy(void* graph) {
    if (!graph) return 0;
    h4b::GraphHandle* h = static_cast<h4b::GraphHandle*>(graph);
    if (h->exec) cudaGraphExecDestroy(h->exec);
    if (h->graph) cudaGraphDestroy(h->graph);
    delete h;
    return 0;
}

extern "C" int h4b_residual_acc(float* x, const int32_t* acc, const float* absmax, const float* w_scales, int n,
                                void* stream) {
    if (!x || !acc || !absmax || !w_scales || n < 1) return H4B_EINVAL;
    h4b::residual_acc_kernel<<<(n + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, acc, absmax, w_scales,
                                                                                           n);
    H4B_CUDA_TRY(cudaGetLastError());
    return 0;
}
