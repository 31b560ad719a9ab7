// Prefill: `count` prompt tokens of one session in one call, through the
// batched GEMMs (the reference feeds a prompt one forward_token at a time,
// cpu_lightspark.py:809-810 and inference_runtime.py:177-181).
//
// Per layer the prompt rows go through the same operations as a decode
// token, M rows at a time: RMSNorm + per-token quantisation, the tensor-core
// int4 GEMM (gemm_tc.cu) for qkv / o / gate-up / down (o and down add into
// x in their epilogue), SwiGLU fused into the quantisation of the down
// input. Attention runs in two launches so no query reads a key that
// another CTA of the same launch is writing:
//   1. prefill_rope_append_kernel: q/k RMSNorm and RoPE for every prompt
//      token and head (the decode kernel's norm_rope), q written back in
//      place, k and v appended to the session's cache at their positions;
//   2. the prompt queries' attention over the cache, by the scratch's
//      attn_kernel and attn_splits:
//      - H4B_PREFILL_ATTN_TENSOR, one split (the default for an fp16 cache,
//        head_dim 128, 4 q heads per kv head): prefill_attention_tc_kernel
//        (prefill_tc.cu), tcgen05 MMAs with split-fp16 operands -- within
//        the fp32 tolerance, not the decode's bits;
//      - otherwise with one split: prefill_attention_block_kernel, blocks of
//        16 queries sharing their K/V sub-tiles, each (query, head) in the
//        decode kernel's order;
//      - more splits: gqa_split_kernel with one batch entry per query on the
//        one cache (batch stride 0), positions p0 + i, no append.
// The exact kernels read back the cache values the first launch stored, in
// the cache precision, exactly as the decode kernel stages its own new key
// and value, so every prompt row equals a chain decode step with the same
// attention splits bit for bit. Only the last row goes through the LM head
// (its logits and greedy token are what forward_token returns).

namespace h4b {

__global__ void prefill_setup_kernel(const int32_t* position, int count, int capacity, int32_t* positions,
                                     unsigned long long* argmax_key) {
    const int p0 = *position;
    const bool fits = p0 >= 0 && p0 + count <= capacity;
    if (!fits && blockIdx.x == 0 && threadIdx.x == 0) report(kStatusBadPosition);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += gridDim.x * blockDim.x)
        positions[i] = fits ? p0 + i : -1;  // -1: the attention kernels skip the row
    if (blockIdx.x == 0 && threadIdx.x == 0) *argmax_key = 0ull;
}

// One warp per (prompt token, head), eight to a CTA: heads [0, q_heads)
// are queries, [q_heads, q_heads + kv_heads) keys (+ the matching value row).
// Batched decode uses it with one row per sequence and row_stride = the
// distance between the sequences' caches.
constexpr int kRopeWarps = 8;

template <typename KV>
__global__ void __launch_bounds__(32 * kRopeWarps) prefill_rope_append_kernel(
    float* qkv, int qkv_stride, int q_heads, int kv_heads, const float* q_norm, const float* k_norm,
    const float* rope_cos, const float* rope_sin, float eps, const int32_t* positions, int count, KV* kcache,
    KV* vcache, long long head_stride, long long time_stride, int capacity, long long row_stride = 0) {
    const int heads = q_heads + kv_heads;
    const long long w = static_cast<long long>(blockIdx.x) * kRopeWarps + (threadIdx.x >> 5);
    if (w >= static_cast<long long>(count) * heads) return;
    const int i = static_cast<int>(w / heads), head = static_cast<int>(w % heads), lane = threadIdx.x & 31;
    const int pos = positions[i];
    if (pos < 0) return;
    if (pos >= capacity) {  // a batch row past its cache (the prefill marks such rows -1)
        if (lane == 0 && head == 0) report(kStatusBadPosition);
        return;
    }
    const float* cs = rope_cos + static_cast<long long>(pos) * (kHeadDim / 2);
    const float* sn = rope_sin + static_cast<long long>(pos) * (kHeadDim / 2);
    float* row = qkv + static_cast<long long>(i) * qkv_stride;
    if (head < q_heads) {
        float4* q = reinterpret_cast<float4*>(row + static_cast<long long>(head) * kHeadDim) + lane;
        *q = norm_rope(*q, q_norm, cs, sn, eps, lane);
        return;
    }
    const int kvh = head - q_heads;
    const float* k = row + static_cast<long long>(q_heads + kvh) * kHeadDim;
    const float* v = row + static_cast<long long>(q_heads + kv_heads + kvh) * kHeadDim;
    const float4 kn = norm_rope(*(reinterpret_cast<const float4*>(k) + lane), k_norm, cs, sn, eps, lane);
    // row_stride: each row its own cache (batched decode), 0: one cache (prefill)
    const long long at = i * row_stride + kvh * head_stride + static_cast<long long>(pos) * time_stride + 4 * lane;
    store4<KV>(kcache + at, kn);
    store4<KV>(vcache + at, *(reinterpret_cast<const float4*>(v) + lane));
}

// Prefill attention with one split per query, for a block of kPrefillQB
// consecutive prompt queries and one kv head per CTA: every K/V sub-tile of
// the block's longest context is staged into shared memory once and folded
// into the running (m, l, o) of every (query, q head) pair that reaches it.
// A pair sees the same sub-tiles, with the same token counts, in the same
// order as gqa_split_kernel gives that query alone with one split, so the
// output is bit for bit the same; only the K/V loads are shared (the block's
// queries have nearly the same context), which cuts L2 traffic by the block
// size. 8 warps; pair j = (query j / G, head j % G) belongs to warp j % 8 and
// keeps its state in registers. G = q heads per kv head (4 for Qwen3-4B).
constexpr int kPrefillQB = 16;
constexpr int kPrefillWarps = 8;
constexpr int kPrefillGroups = 4;

template <typename KV>
__host__ __device__ constexpr int prefill_block_smem_bytes() {
    return 2 * kSubTile * kv_row_stride<KV>() * static_cast<int>(sizeof(KV)) +
           kPrefillQB * kPrefillGroups * kHeadDim * 4;
}

template <typename KV>
__global__ void __launch_bounds__(kPrefillWarps * 32) prefill_attention_block_kernel(
    const float* qkv, int qkv_stride, const KV* kcache, const KV* vcache, long long head_stride,
    long long time_stride, const int32_t* positions, int count, float* out, int out_stride) {
    constexpr int groups = kPrefillGroups;
    constexpr int kPrefillMaxPairs = kPrefillQB * groups / kPrefillWarps;
    extern __shared__ __align__(16) uint8_t pb_smem[];
    KV* ks = reinterpret_cast<KV*>(pb_smem);
    KV* vs = ks + kSubTile * kv_row_stride<KV>();
    float* qs = reinterpret_cast<float*>(vs + kSubTile * kv_row_stride<KV>());  // [qb][groups][d]
    // the longest contexts (the last query blocks) first, so the tail is short
    const int kvh = blockIdx.x, q0 = (gridDim.y - 1 - blockIdx.y) * kPrefillQB;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nq = min(kPrefillQB, count - q0);
    const int pairs = nq * groups;
    const KV* kc = kcache + kvh * head_stride;
    const KV* vc = vcache + kvh * head_stride;
    // the block's queries (already normalised and rotated by the append kernel)
    for (int i = threadIdx.x; i < pairs * (kHeadDim / 4); i += blockDim.x) {
        const int pair = i / (kHeadDim / 4), piece = i % (kHeadDim / 4);
        const int qi = pair / groups, h = pair % groups;
        const float4* src = reinterpret_cast<const float4*>(
            qkv + static_cast<long long>(q0 + qi) * qkv_stride + static_cast<long long>(kvh * groups + h) * kHeadDim);
        reinterpret_cast<float4*>(qs + pair * kHeadDim)[piece] = src[piece];
    }
    int max_ctx = 0;
    for (int qi = 0; qi < nq; ++qi) max_ctx = max(max_ctx, positions[q0 + qi] + 1);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(kHeadDim)));
    float m[kPrefillMaxPairs], l[kPrefillMaxPairs];
    float4 o[kPrefillMaxPairs];
#pragma unroll
    for (int j = 0; j < kPrefillMaxPairs; ++j) {
        m[j] = -INFINITY;
        l[j] = 0.f;
        o[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    #pragma unroll 1
    for (int base = 0; base < max_ctx; base += kSubTile) {
        const int n_max = min(kSubTile, max_ctx - base);
        __syncthreads();  // the previous sub-tile (and, first, the queries) are settled
        stage_subtile<KV>(kc, vc, time_stride, base, n_max, -1, ks, vs, threadIdx.x, blockDim.x);
        async_copy_wait_all();
        __syncthreads();
#pragma unroll
        for (int j = 0; j < kPrefillMaxPairs; ++j) {
            const int pair = warp + kPrefillWarps * j;
            if (pair >= pairs) continue;
            const int ctx = positions[q0 + pair / groups] + 1;  // 0 for a row that does not fit
            if (base >= ctx) continue;
            attend_subtile<KV>(qs + pair * kHeadDim, ks, vs, min(kSubTile, ctx - base), scale, lane, m[j], l[j], o[j]);
        }
    }
#pragma unroll
    for (int j = 0; j < kPrefillMaxPairs; ++j) {
        const int pair = warp + kPrefillWarps * j;
        if (pair >= pairs) continue;
        const int qi = pair / groups, h = pair % groups;
        if (positions[q0 + qi] < 0) continue;
        const float inv = __fdiv_rn(1.0f, l[j]);
        const float4 r = make_float4(o[j].x * inv, o[j].y * inv, o[j].z * inv, o[j].w * inv);
        *reinterpret_cast<float4*>(out + static_cast<long long>(q0 + qi) * out_stride +
                                   static_cast<long long>(kvh * groups + h) * kHeadDim + 4 * lane) = r;
    }
}

// Shared-memory opt-in of the block kernels above 48 KB, per device,
// recording only a success.
static int prefill_block_opt_in() {
    static std::atomic<bool> opted_in[kMaxDevices];
    int dev = 0;
    H4B_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return H4B_EUNSUPPORTED;
    if (!opted_in[dev].load(std::memory_order_acquire)) {
        H4B_CUDA_TRY(cudaFuncSetAttribute(prefill_attention_block_kernel<float>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, prefill_block_smem_bytes<float>()));
        H4B_CUDA_TRY(cudaFuncSetAttribute(prefill_attention_block_kernel<__half>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          prefill_block_smem_bytes<__half>()));
        opted_in[dev].store(true, std::memory_order_release);
    }
    return 0;
}

__global__ void prefill_finish_kernel(const unsigned long long* argmax_key, int32_t* next_token, int32_t* token,
                                      int32_t* position, int count) {
    if (threadIdx.x == 0) {
        const int32_t id = static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(*argmax_key & 0xFFFFFFFFull));
        *next_token = id;
        if (token) *token = id;
        *position += count;
    }
}

int validate_prefill(const h4b_model* m, const h4b_state* s, const h4b_prefill_scratch* p, int count) {
    int rc = validate(m, s);
    if (rc) return rc;
    if (!p || count < 1 || count > p->max_tokens || p->attn_queries < 1) return H4B_EINVAL;
    if (p->attn_splits < 1 || p->attn_splits > 64) return H4B_EINVAL;
    const void* required[] = {p->x, p->x8, p->act_scale, p->act_sum, p->qkv, p->attended, p->gate_up, p->act,
                              p->proj, p->tokens, p->positions};
    for (const void* q : required)
        if (!q || (reinterpret_cast<uintptr_t>(q) & 15)) return H4B_EINVAL;
    if (p->attn_splits > 1 && (!p->attn_partials || !p->attn_counters)) return H4B_EINVAL;
    if (p->attn_kernel != H4B_PREFILL_ATTN_EXACT && p->attn_kernel != H4B_PREFILL_ATTN_TENSOR) return H4B_EINVAL;
    return 0;
}

// The parts of a prefill layer, shared by the single-GPU loop (prefill)
// and the tensor-parallel stages (prefill_tp_stage).
struct PrefillRun {
    const h4b_model* m;
    const h4b_state* s;
    const h4b_prefill_scratch* p;
    int count;
    cudaStream_t stream;

    int gemm(const uint8_t* w, const float* ws, float* out, int rows, int width, int32_t* out_i32 = nullptr,
             bool residual = false) const {
        GemmArgs g{p->x8, p->act_scale, p->act_sum, w, ws, out, count, rows, width};
        g.out_i32 = out_i32;
        g.residual = residual;
        return launch_int4_gemm(g, stream);
    }
    // RMSNorm, quantisation and the gate/up GEMM, then SwiGLU fused into the
    // quantisation of its rows for the down projection.
    int mlp_quantised(int l) const {
        const int H = m->hidden, I = m->intermediate;
        int rc;
        if ((rc = norm_quant(m->norm_post + static_cast<size_t>(l) * H))) return rc;
        if ((rc = gemm(m->w_gate_up + static_cast<size_t>(l) * 2 * I * (H / 2),
                       m->s_gate_up + static_cast<size_t>(l) * 2 * I, p->gate_up, 2 * I, H)))
            return rc;
        return launch_quantize_rows<true>(p->gate_up, I, count, p->x8, p->act_scale, p->act_sum, p->act, stream);
    }
    int norm_quant(const float* gamma) const {
        return launch_rmsnorm_quant(p->x, gamma, m->eps, m->hidden, count, p->x8, p->act_scale, p->act_sum, stream);
    }
    int setup(const uint8_t* table, const float* table_scales, int table_vocab) const {
        prefill_setup_kernel<<<std::min((count + 255) / 256, 148), 256, 0, stream>>>(s->position, count, s->capacity,
                                                                                   p->positions, s->argmax_key);
        batch_embed_kernel<<<count, 256, 0, stream>>>(p->tokens, table, table_scales, table_vocab, m->hidden, p->x);
        H4B_CUDA_TRY(cudaGetLastError());
        return 0;
    }
    // RMSNorm, quantisation, the qkv GEMM, q/k norm + RoPE + K/V append and
    // attention of every prompt row: p->attended.
    int attention_block(int l) const {
        const int H = m->hidden, d = m->head_dim;
        const int q_size = m->heads * d, kv_size = m->kv_heads * d, qkv_rows = q_size + 2 * kv_size;
        const size_t kv_layer = static_cast<size_t>(m->kv_heads) * s->capacity * d;  // elements
        const size_t eb = s->kv_dtype == 0 ? 4 : 2;
        int rc;
        if ((rc = norm_quant(m->norm_in + static_cast<size_t>(l) * H))) return rc;
        if ((rc = gemm(m->w_qkv + static_cast<size_t>(l) * qkv_rows * (H / 2), m->s_qkv + static_cast<size_t>(l) * qkv_rows,
                       p->qkv, qkv_rows, H)))
            return rc;
        char* kc = static_cast<char*>(s->k_cache) + l * kv_layer * eb;
        char* vc = static_cast<char*>(s->v_cache) + l * kv_layer * eb;
        const long long pairs = static_cast<long long>(count) * (m->heads + m->kv_heads);
        const int rope_grid = static_cast<int>((pairs + kRopeWarps - 1) / kRopeWarps);
        const long long head_stride = static_cast<long long>(s->capacity) * d;
        if (s->kv_dtype == 0)
            prefill_rope_append_kernel<float><<<rope_grid, 32 * kRopeWarps, 0, stream>>>(
                p->qkv, qkv_rows, m->heads, m->kv_heads, m->norm_q + static_cast<size_t>(l) * d,
                m->norm_k + static_cast<size_t>(l) * d, m->rope_cos, m->rope_sin, m->eps, p->positions, count,
                reinterpret_cast<float*>(kc), reinterpret_cast<float*>(vc), head_stride, d, s->capacity);
        else
            prefill_rope_append_kernel<__half><<<rope_grid, 32 * kRopeWarps, 0, stream>>>(
                p->qkv, qkv_rows, m->heads, m->kv_heads, m->norm_q + static_cast<size_t>(l) * d,
                m->norm_k + static_cast<size_t>(l) * d, m->rope_cos, m->rope_sin, m->eps, p->positions, count,
                reinterpret_cast<__half*>(kc), reinterpret_cast<__half*>(vc), head_stride, d, s->capacity);
        H4B_CUDA_TRY(cudaGetLastError());
        return attention_only(l);
    }
    // The prompt rows' attention of layer l alone (q rows in p->qkv, already
    // normalised and rotated; K/V appended): p->attended.
    int attention_only(int l) const {
        const int d = m->head_dim;
        const int q_size = m->heads * d, kv_size = m->kv_heads * d, qkv_rows = q_size + 2 * kv_size;
        const size_t kv_layer = static_cast<size_t>(m->kv_heads) * s->capacity * d;  // elements
        const size_t eb = s->kv_dtype == 0 ? 4 : 2;
        char* kc = static_cast<char*>(s->k_cache) + l * kv_layer * eb;
        char* vc = static_cast<char*>(s->v_cache) + l * kv_layer * eb;
        const long long head_stride = static_cast<long long>(s->capacity) * d;
        int rc;
        if (p->attn_splits == 1 && p->attn_kernel == H4B_PREFILL_ATTN_TENSOR &&
            prefill_tc_supported(s->kv_dtype, d, m->heads / m->kv_heads))
            return launch_prefill_attention_tc(p->qkv, qkv_rows, reinterpret_cast<const __half*>(kc),
                                               reinterpret_cast<const __half*>(vc), m->kv_heads, s->capacity,
                                               p->positions, count, p->attended, q_size, stream);
        if (p->attn_splits == 1 && m->heads / m->kv_heads == kPrefillGroups) {
            // one split per query: query blocks share their K/V sub-tiles
            int rc2 = prefill_block_opt_in();
            if (rc2) return rc2;
            const dim3 grid(m->kv_heads, (count + kPrefillQB - 1) / kPrefillQB);
            if (s->kv_dtype == 0)
                prefill_attention_block_kernel<float><<<grid, kPrefillWarps * 32, prefill_block_smem_bytes<float>(),
                                                         stream>>>(
                    p->qkv, qkv_rows, reinterpret_cast<const float*>(kc), reinterpret_cast<const float*>(vc),
                    head_stride, d, p->positions, count, p->attended, q_size);
            else
                prefill_attention_block_kernel<__half><<<grid, kPrefillWarps * 32, prefill_block_smem_bytes<__half>(),
                                                          stream>>>(
                    p->qkv, qkv_rows, reinterpret_cast<const __half*>(kc), reinterpret_cast<const __half*>(vc),
                    head_stride, d, p->positions, count, p->attended, q_size);
            H4B_CUDA_TRY(cudaGetLastError());
            return 0;
        }
        for (int c0 = 0; c0 < count; c0 += p->attn_queries) {
            const int n = std::min(p->attn_queries, count - c0);
            AttnArgs a = {};
            a.q = p->qkv + static_cast<size_t>(c0) * qkv_rows;
            a.q_batch_stride = qkv_rows;
            a.eps = m->eps;
            a.kcache = kc; a.vcache = vc;
            a.head_stride = head_stride;
            a.time_stride = d;
            a.batch_stride = 0;
            a.position = p->positions + c0; a.capacity = s->capacity;
            a.groups = m->heads / m->kv_heads; a.kv_heads = m->kv_heads; a.splits = p->attn_splits;
            a.partials = p->attn_partials; a.counters = p->attn_counters;
            a.out = p->attended + static_cast<size_t>(c0) * q_size; a.out_batch_stride = q_size;
            if ((rc = launch_attention(a, s->kv_dtype, n, stream, false))) return rc;
        }
        return 0;
    }
    // RMSNorm, quantisation, the gate/up GEMM and SwiGLU: p->act.
    int mlp_block(int l) const {
        const int H = m->hidden, I = m->intermediate;
        int rc;
        if ((rc = norm_quant(m->norm_post + static_cast<size_t>(l) * H))) return rc;
        if ((rc = gemm(m->w_gate_up + static_cast<size_t>(l) * 2 * I * (H / 2),
                       m->s_gate_up + static_cast<size_t>(l) * 2 * I, p->gate_up, 2 * I, H)))
            return rc;
        const long long n_act = static_cast<long long>(count) * I;
        batch_swiglu_kernel<<<static_cast<int>((n_act + 255) / 256), 256, 0, stream>>>(p->gate_up, I, count, p->act);
        H4B_CUDA_TRY(cudaGetLastError());
        return 0;
    }
    // The last prompt row: final RMSNorm, LM head, greedy token (the decode stages).
    int finish() const {
        H4B_CUDA_TRY(cudaMemcpyAsync(s->x, p->x + static_cast<size_t>(count - 1) * m->hidden,
                                     sizeof(float) * m->hidden, cudaMemcpyDeviceToDevice, stream));
        int rc;
        if ((rc = launch_stage(m, s, STAGE_LM_HEAD, 0, stream, false))) return rc;
        prefill_finish_kernel<<<1, 32, 0, stream>>>(s->argmax_key, s->next_token, s->token, s->position, count);
        H4B_CUDA_TRY(cudaGetLastError());
        return 0;
    }
};

int prefill(const h4b_model* m, const h4b_state* s, const h4b_prefill_scratch* p, int count, cudaStream_t stream) {
    int rc = validate_prefill(m, s, p, count);
    if (rc) return rc;
    const int H = m->hidden, I = m->intermediate, q_size = m->heads * m->head_dim;
    const PrefillRun r{m, s, p, count, stream};
    if ((rc = r.setup(m->w_embed, m->s_embed, m->vocab))) return rc;
    // The residual adds ride in the o / down GEMM epilogues (x + proj, in
    // that order), SwiGLU in the quantisation of its rows: the same
    // operations as the separate kernels, bit for bit.
    for (int l = 0; l < m->layers; ++l) {
        if ((rc = r.attention_block(l))) return rc;
        if ((rc = launch_quantize_rows<false>(p->attended, q_size, count, p->x8, p->act_scale, p->act_sum, nullptr,
                                              stream)))
            return rc;
        if ((rc = r.gemm(m->w_o + static_cast<size_t>(l) * H * (q_size / 2), m->s_o + static_cast<size_t>(l) * H, p->x,
                         H, q_size, nullptr, true)))
            return rc;
        if ((rc = r.mlp_quantised(l))) return rc;
        if ((rc = r.gemm(m->w_down + static_cast<size_t>(l) * H * (I / 2), m->s_down + static_cast<size_t>(l) * H, p->x,
                         H, I, nullptr, true)))
            return rc;
    }
    return r.finish();
}

// ---- tensor-parallel prefill stages ------------------------------------------
// Each rank holds a slice (its heads, its MLP units, K-slices of o and down,
// its vocabulary rows); x is replicated. Between the stages the caller runs
// the cross-rank reductions: a MAX over `absmax` after stages 1 and 3, an
// exact int32 SUM over `acc` after stages 2 and 4.

__global__ void __launch_bounds__(256) row_absmax_kernel(const float* v, int K, float* out) {
    __shared__ float red[8];
    const float* row = v + static_cast<size_t>(blockIdx.x) * K;
    float mx = 0.f;
    for (int i = threadIdx.x; i < K; i += blockDim.x) mx = fmaxf(mx, fabsf(row[i]));
    mx = warp_max(mx);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    if (threadIdx.x == 0) {
        float m = red[0];
        for (int w = 1; w < 8; ++w) m = fmaxf(m, red[w]);
        out[blockIdx.x] = m;
    }
}

// x[m][r] += float(acc[m][r]) * act_scale[m] * w_scale[r] (the GEMM epilogue
// order, then the residual add).
__global__ void residual_rows_kernel(float* x, const int32_t* acc, const float* act_scale, const float* w_scale,
                                     int rows, int H) {
    const long long n = static_cast<long long>(rows) * H;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int mrow = static_cast<int>(i / H), r = static_cast<int>(i - static_cast<long long>(mrow) * H);
        x[i] = __fadd_rn(x[i], __fmul_rn(__fmul_rn(static_cast<float>(acc[i]), act_scale[mrow]), w_scale[r]));
    }
}

int prefill_tp_stage(const h4b_model* m, const h4b_state* s, const h4b_prefill_scratch* p, int count, int layer,
                     int stage, const uint8_t* table, const float* table_scales, int table_vocab, float* absmax,
                     int32_t* acc, cudaStream_t stream) {
    int rc = validate_prefill(m, s, p, count);
    if (rc) return rc;
    if (!absmax || !acc) return H4B_EINVAL;
    if (stage >= 1 && stage <= 5 && (layer < 0 || layer >= m->layers)) return H4B_EINVAL;
    const int H = m->hidden, I = m->intermediate, q_size = m->heads * m->head_dim;
    const size_t l = static_cast<size_t>(layer);
    const PrefillRun r{m, s, p, count, stream};
    const int grid = std::max(1, std::min(static_cast<int>((static_cast<long long>(count) * H + 255) / 256),
                                          8 * sm_count()));
    switch (stage) {
        case 0:
            if (!table || !table_scales || table_vocab < 1) return H4B_EINVAL;
            return r.setup(table, table_scales, table_vocab);
        case 1:
            if ((rc = r.attention_block(layer))) return rc;
            row_absmax_kernel<<<count, 256, 0, stream>>>(p->attended, q_size, absmax);
            break;
        case 2:
            quantize_rows_kernel<<<count, 256, 0, stream>>>(p->attended, q_size, p->x8, p->act_scale, p->act_sum,
                                                            absmax);
            H4B_CUDA_TRY(cudaGetLastError());
            return r.gemm(m->w_o + l * H * (q_size / 2), m->s_o + l * H, p->proj, H, q_size, acc);
        case 3:
            residual_rows_kernel<<<grid, 256, 0, stream>>>(p->x, acc, p->act_scale, m->s_o + l * H, count, H);
            H4B_CUDA_TRY(cudaGetLastError());
            if ((rc = r.mlp_block(layer))) return rc;
            row_absmax_kernel<<<count, 256, 0, stream>>>(p->act, I, absmax);
            break;
        case 4:
            quantize_rows_kernel<<<count, 256, 0, stream>>>(p->act, I, p->x8, p->act_scale, p->act_sum, absmax);
            H4B_CUDA_TRY(cudaGetLastError());
            return r.gemm(m->w_down + l * H * (I / 2), m->s_down + l * H, p->proj, H, I, acc);
        case 5:
            residual_rows_kernel<<<grid, 256, 0, stream>>>(p->x, acc, p->act_scale, m->s_down + l * H, count, H);
            break;
        case 6:
            return r.finish();
        default:
            return H4B_EINVAL;
    }
    H4B_CUDA_TRY(cudaGetLastError());
    return 0;
}

}  // namespace h4b

extern "C" int h4b_prefill(const h4b_model* model, const h4b_state* state, const h4b_prefill_scratch* scratch,
                           int count, void* stream) {
    return h4b::prefill(model, state, scratch, count, static_cast<cudaStream_t>(stream));
}

extern "C" int h4b_prefill_attention(const h4b_model* model, const h4b_state* state,
                                     const h4b_prefill_scratch* scratch, int count, int layer, void* stream) {
    int rc = h4b::validate_prefill(model, state, scratch, count);
    if (rc) return rc;
    if (layer < 0 || layer >= model->layers) return H4B_EINVAL;
    const h4b::PrefillRun r{model, state, scratch, count, static_cast<cudaStream_t>(stream)};
    return r.attention_only(layer);
}

extern "C" int h4b_prefill_tp_stage(const h4b_model* model, const h4b_state* state, const h4b_prefill_scratch* scratch,
                                    int count, int layer, int stage, const uint8_t* table, const float* table_scales,
                                    int table_vocab, float* absmax, int32_t* acc, void* stream) {
    return h4b::prefill_tp_stage(model, state, scratch, count, layer, stage, table, table_scales, table_vocab, absmax,
                                 acc, static_cast<cudaStream_t>(stream));
}
