// Batched decode: B sequences advance one token each per call
// (LiteSparkQwen.forward_token, cpu_lightspark.py:424-468, for a batch; the
// reference has no batched path). The body projections run as tensor-core
// GEMMs (gemm.cu) over the B activations; attention runs the split-K kernel
// with its batch dimension (each sequence has its own position and KV
// cache). Every row follows the single-token arithmetic exactly: RMSNorm in
// the GEMV prologue's 256-lane order, per-token absmax quantisation, exact
// int32 sums with the float(acc) * act_scale * w_scale epilogue, the same
// attention kernel, residual adds and SwiGLU -- so each sequence's logits
// equal what the one-token chain gives it.

namespace h4b {

// Embedding rows (cpu_lightspark.py:341-349): one CTA per sequence.
__global__ void batch_embed_kernel(const int32_t* tokens, const uint8_t* table, const float* scales, int vocab, int H,
                                   float* x) {
    const int b = blockIdx.x;
    const int token = tokens[b];
    const bool ok = token >= 0 && token < vocab;
    if (!ok && threadIdx.x == 0) report(kStatusBadToken);
    const float scale = ok ? scales[token] : 0.f;
    const uint8_t* row = table + static_cast<size_t>(ok ? token : 0) * (H >> 1);
    float* out = x + static_cast<size_t>(b) * H;
    for (int j = threadIdx.x; j < (H >> 1); j += blockDim.x) {
        const int8_t byte = static_cast<int8_t>(row[j]);
        out[2 * j] = ok ? __fmul_rn(static_cast<float>(static_cast<int8_t>(byte << 4) >> 4), scale) : 0.f;
        out[2 * j + 1] = ok ? __fmul_rn(static_cast<float>(byte >> 4), scale) : 0.f;
    }
}

// RMSNorm + per-token quantisation of one row per CTA (256 threads), in the
// GEMV prologue's order: thread p sums groups p, p + 256, ... of 8 values
// with fmaf, warps are butterfly-summed and added in order; x8 is written in
// plain k order for the GEMM, with the row's int8 sum and dequant scale.
__global__ void __launch_bounds__(256) batch_rmsnorm_quant_kernel(const float* x, const float* gamma, float eps, int H,
                                                                  int8_t* x8, float* act_scale, int32_t* act_sum) {
    __shared__ float red[32];
    __shared__ int ired[8];
    const int b = blockIdx.x, tid = threadIdx.x;
    const float* row = x + static_cast<size_t>(b) * H;
    const int groups = H >> 3;
    float ss = 0.f;
    for (int g = tid; g < groups; g += 256) {
        float v[8];
        load8(row + 8 * g, v);
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = __fmaf_rn(v[e], v[e], ss);
    }
    ss = group_sum(ss, red, 8, 1);
    const float mean = __fdiv_rn(ss, static_cast<float>(H));
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    float local = 0.f;
    for (int g = tid; g < groups; g += 256) {
        float v[8], gm[8];
        load8(row + 8 * g, v);
        load8(gamma + 8 * g, gm);
#pragma unroll
        for (int e = 0; e < 8; ++e) local = fmaxf(local, fabsf(__fmul_rn(__fmul_rn(v[e], inv), gm[e])));
    }
    const float m = group_max(local, red, 8, 1);
    const float qs = quant_multiplier(m);
    int8_t* out = x8 + static_cast<size_t>(b) * H;
    int sum = 0;
    for (int g = tid; g < groups; g += 256) {
        float v[8], gm[8];
        load8(row + 8 * g, v);
        load8(gamma + 8 * g, gm);
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const int q = quantize_one(__fmul_rn(__fmul_rn(v[e], inv), gm[e]), qs);
            sum += q;
            if (e < 4) lo |= static_cast<uint32_t>(q & 0xFF) << (8 * e);
            else hi |= static_cast<uint32_t>(q & 0xFF) << (8 * (e - 4));
        }
        *reinterpret_cast<uint2*>(out + 8 * g) = make_uint2(lo, hi);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if ((tid & 31) == 0) ired[tid >> 5] = sum;
    __syncthreads();
    if (tid == 0) {
        int t = 0;
        for (int w = 0; w < 8; ++w) t += ired[w];
        act_sum[b] = t;
        act_scale[b] = dequant_scale(m);
    }
}

// batch_rmsnorm_quant_kernel's result, bit for bit (each thread keeps the
// same groups in the same order, and the block reductions are the same), with
// the thread's kG groups of 8 held in registers: one read of the row instead
// of three. With pending residual sums (the o / down GEMM's split-K sums left
// in pend.acc), it first does the finalize kernel's residual step on its row,
// x = x + float(acc) * as * ws in that order, stores x and zeroes acc.
template <int kG>
__global__ void __launch_bounds__(256) batch_rmsnorm_quant_reg_kernel(float* x, const float* gamma, float eps,
                                                                      int H, int8_t* x8, float* act_scale,
                                                                      int32_t* act_sum, PendingSums pend) {
    __shared__ float red[32];
    __shared__ int ired[8];
    const int b = blockIdx.x, tid = threadIdx.x;
    float* row = x + static_cast<size_t>(b) * H;
    const int groups = H >> 3;
    // read before this row's scale is overwritten at the end (after the barriers)
    int32_t* prow = pend.acc ? pend.acc + static_cast<size_t>(b) * pend.stride : nullptr;
    const float pas = pend.acc ? pend.as[b] : 0.f;
    float v[kG][8], gm[kG][8];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < kG; ++k) {
        const int g = tid + 256 * k;
        if (g < groups) {
            load8(row + 8 * g, v[k]);
            load8(gamma + 8 * g, gm[k]);
            if (prow) {
                int4* cell = reinterpret_cast<int4*>(prow + 8 * g);
                const int4 s0 = cell[0], s1 = cell[1];
                float w[8];
                load8(pend.ws + 8 * g, w);
                const int sum[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
                for (int e = 0; e < 8; ++e) v[k][e] = __fadd_rn(v[k][e], pending_value(sum[e], pas, w[e]));
                float4* out = reinterpret_cast<float4*>(row + 8 * g);
                out[0] = make_float4(v[k][0], v[k][1], v[k][2], v[k][3]);
                out[1] = make_float4(v[k][4], v[k][5], v[k][6], v[k][7]);
                cell[0] = make_int4(0, 0, 0, 0);
                cell[1] = make_int4(0, 0, 0, 0);
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) ss = __fmaf_rn(v[k][e], v[k][e], ss);
        }
    }
    ss = group_sum(ss, red, 8, 1);
    const float mean = __fdiv_rn(ss, static_cast<float>(H));
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    float local = 0.f;
#pragma unroll
    for (int k = 0; k < kG; ++k) {
        if (tid + 256 * k < groups) {
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                v[k][e] = __fmul_rn(__fmul_rn(v[k][e], inv), gm[k][e]);
                local = fmaxf(local, fabsf(v[k][e]));
            }
        }
    }
    const float m = group_max(local, red, 8, 1);
    const float qs = quant_multiplier(m);
    int8_t* out = x8 + static_cast<size_t>(b) * H;
    int sum = 0;
#pragma unroll
    for (int k = 0; k < kG; ++k) {
        const int g = tid + 256 * k;
        if (g < groups) {
            uint32_t lo = 0, hi = 0;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const int q = quantize_one(v[k][e], qs);
                sum += q;
                if (e < 4) lo |= static_cast<uint32_t>(q & 0xFF) << (8 * e);
                else hi |= static_cast<uint32_t>(q & 0xFF) << (8 * (e - 4));
            }
            *reinterpret_cast<uint2*>(out + 8 * g) = make_uint2(lo, hi);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if ((tid & 31) == 0) ired[tid >> 5] = sum;
    __syncthreads();
    if (tid == 0) {
        int t = 0;
        for (int w = 0; w < 8; ++w) t += ired[w];
        act_sum[b] = t;
        act_scale[b] = dequant_scale(m);
    }
}

// RMSNorm + per-row quantisation of `rows` rows of H (the register kernel
// when a thread's share fits, else the three-pass kernel).
inline bool rmsnorm_quant_reg_fits(int H) { return H % 8 == 0 && (H / 8 + 255) / 256 <= 4; }

// `pend` (the register kernel only): the pending residual sums of the
// projection that produced x, applied to x first.
int launch_rmsnorm_quant(float* x, const float* gamma, float eps, int H, int rows, int8_t* x8,
                         float* act_scale, int32_t* act_sum, cudaStream_t stream, PendingSums pend = {}) {
    const int per = (H / 8 + 255) / 256;
    if (pend.acc && (!rmsnorm_quant_reg_fits(H) || pend.stride % 4 != 0 ||
                     ((reinterpret_cast<uintptr_t>(pend.acc) | reinterpret_cast<uintptr_t>(pend.ws) |
                       reinterpret_cast<uintptr_t>(x)) & 15) != 0))
        return H4B_EUNSUPPORTED;
    if (H % 8 == 0 && per <= 1)
        batch_rmsnorm_quant_reg_kernel<1><<<rows, 256, 0, stream>>>(x, gamma, eps, H, x8, act_scale, act_sum, pend);
    else if (H % 8 == 0 && per == 2)
        batch_rmsnorm_quant_reg_kernel<2><<<rows, 256, 0, stream>>>(x, gamma, eps, H, x8, act_scale, act_sum, pend);
    else if (H % 8 == 0 && per <= 4)
        batch_rmsnorm_quant_reg_kernel<4><<<rows, 256, 0, stream>>>(x, gamma, eps, H, x8, act_scale, act_sum, pend);
    else
        batch_rmsnorm_quant_kernel<<<rows, 256, 0, stream>>>(x, gamma, eps, H, x8, act_scale, act_sum);
    H4B_CUDA_TRY(cudaGetLastError());
    return 0;
}

// SwiGLU over rows laid out like the fused gate/up weight (blocks of 4 gate
// rows then the 4 matching up rows): act = gate / (1 + exp(-gate)) * up.
__global__ void batch_swiglu_kernel(const float* gate_up, int I, int B, float* act) {
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<long long>(B) * I) return;
    const long long b = i / I;
    const int p = static_cast<int>(i % I);
    const int blk = p / kSwigluBlock, j = p % kSwigluBlock;
    const float* row = gate_up + b * 2 * I;
    const float g = row[2 * kSwigluBlock * blk + j], u = row[2 * kSwigluBlock * blk + kSwigluBlock + j];
    act[i] = swiglu_one(g, u);
}

// Greedy token per row (first maximum, numpy argmax semantics).
__global__ void __launch_bounds__(1024) batch_argmax_kernel(const float* logits, int V, int32_t* out) {
    __shared__ unsigned long long keys[32];
    const float* row = logits + static_cast<size_t>(blockIdx.x) * V;
    unsigned long long best = 0ull;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
        const unsigned long long k = argmax_key(row[i], static_cast<uint32_t>(i));
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
        for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) best = keys[w] > best ? keys[w] : best;
        out[blockIdx.x] = static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(best & 0xFFFFFFFFull));
    }
}

__global__ void batch_advance_kernel(int32_t* positions, int B) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < B) positions[b] += 1;
}

int validate_batch(const h4b_model* m, const h4b_batch_state* s) {
    if (!m || !s || s->batch < 1) return H4B_EINVAL;
    if (m->head_dim != kHeadDim) return H4B_EUNSUPPORTED;
    if (m->layers < 1 || m->kv_heads < 1 || m->heads % m->kv_heads) return H4B_EINVAL;
    if (m->heads / m->kv_heads > kMaxGroups) return H4B_EUNSUPPORTED;
    const int q_size = m->heads * m->head_dim, kv_size = m->kv_heads * m->head_dim;
    // GEMM tiles: 128 output rows, 64-wide k steps; RMSNorm groups of 8
    const int rows[] = {q_size + 2 * kv_size, m->hidden, 2 * m->intermediate, m->vocab};
    for (int r : rows)
        if (r % kGemmRows) return H4B_EUNSUPPORTED;
    const int widths[] = {m->hidden, q_size, m->intermediate};
    for (int w : widths)
        if (w % kGemmK) return H4B_EUNSUPPORTED;
    if (m->intermediate % kSwigluBlock) return H4B_EUNSUPPORTED;
    if (s->capacity < 1 || s->capacity > m->max_pos) return H4B_EINVAL;
    if (s->kv_dtype != 0 && s->kv_dtype != 1) return H4B_EINVAL;
    if (s->attn_splits < 1 || s->attn_splits > 64) return H4B_EINVAL;
    if (s->attn_kernel != H4B_BATCH_ATTN_EXACT && s->attn_kernel != H4B_BATCH_ATTN_TENSOR) return H4B_EINVAL;
    if (s->gemm_acc_width < 0) return H4B_EINVAL;
    const void* required[] = {m->w_qkv, m->s_qkv, m->w_o, m->s_o, m->w_gate_up, m->s_gate_up, m->w_down, m->s_down,
                              m->w_embed, m->s_embed, m->norm_in, m->norm_post, m->norm_q, m->norm_k, m->norm_final,
                              m->rope_cos, m->rope_sin, s->k_cache, s->v_cache, s->positions, s->tokens,
                              s->next_tokens, s->x, s->x8, s->act_scale, s->act_sum, s->qkv, s->attended, s->proj,
                              s->gate_up, s->act, s->logits};
    for (const void* p : required)
        if (!p || (reinterpret_cast<uintptr_t>(p) & 15)) return H4B_EINVAL;
    if (s->attn_splits > 1 && (!s->attn_partials || !s->attn_counters)) return H4B_EINVAL;
    return 0;
}

// Layer l's attention for every sequence of the batch: qk-RMSNorm, RoPE,
// append at each sequence's position, split-K GQA over its own cache.
// decode_tc.cu
int launch_batch_attention_tc(const h4b_model* m, const h4b_batch_state* s, int l, cudaStream_t stream);
bool batch_tc_supported(int kv_dtype, int head_dim, int groups);

int batch_attention(const h4b_model* m, const h4b_batch_state* s, int l, cudaStream_t stream) {
    if (s->attn_kernel == H4B_BATCH_ATTN_TENSOR && batch_tc_supported(s->kv_dtype, m->head_dim, m->heads / m->kv_heads))
        return launch_batch_attention_tc(m, s, l, stream);
    const int d = m->head_dim, q_size = m->heads * d, kv_size = m->kv_heads * d, qkv_rows = q_size + 2 * kv_size;
    const size_t kv_layer = static_cast<size_t>(m->kv_heads) * s->capacity * d;  // elements
    AttnArgs a = {};
    a.q = s->qkv; a.knew = s->qkv + q_size; a.vnew = s->qkv + q_size + kv_size;
    a.q_batch_stride = qkv_rows;
    a.q_norm = m->norm_q + static_cast<size_t>(l) * d;
    a.k_norm = m->norm_k + static_cast<size_t>(l) * d;
    a.rope_cos = m->rope_cos; a.rope_sin = m->rope_sin; a.eps = m->eps;
    const size_t eb = s->kv_dtype == 0 ? 4 : 2;
    a.kcache = static_cast<char*>(s->k_cache) + l * kv_layer * eb;
    a.vcache = static_cast<char*>(s->v_cache) + l * kv_layer * eb;
    a.head_stride = static_cast<long long>(s->capacity) * d;
    a.time_stride = d;
    a.batch_stride = static_cast<long long>(m->layers) * kv_layer;
    a.position = s->positions; a.capacity = s->capacity;
    a.groups = m->heads / m->kv_heads; a.kv_heads = m->kv_heads; a.splits = s->attn_splits;
    a.partials = s->attn_partials; a.counters = s->attn_counters;
    a.out = s->attended; a.out_batch_stride = q_size; a.absmax_out = nullptr;
    return launch_attention(a, s->kv_dtype, s->batch, stream, false);
}

int decode_batch(const h4b_model* m, const h4b_batch_state* s, cudaStream_t stream) {
    int rc = validate_batch(m, s);
    if (rc) return rc;
    const int B = s->batch, H = m->hidden, I = m->intermediate, d = m->head_dim;
    const int q_size = m->heads * d, kv_size = m->kv_heads * d, qkv_rows = q_size + 2 * kv_size;
    // split-K / stream-K room: gemm_acc holds B rows of gemm_acc_width int32
    const int acc_rows = s->gemm_acc_width > 0
                             ? s->gemm_acc_width
                             : std::max(m->heads * m->head_dim + 2 * m->kv_heads * m->head_dim, m->hidden);
    // `deferred` (o, down, gate/up): a split GEMM leaves its int32 sums
    // pending in gemm_acc instead of running the finalize kernel, and the
    // next kernel -- the RMSNorm quantisation after o / down, the SwiGLU
    // quantisation after gate/up -- applies them with the same arithmetic
    auto gemm = [&](const uint8_t* w, const float* ws, float* out, int rows, int width, bool residual = false,
                    bool* deferred = nullptr) {
        GemmArgs g{s->x8, s->act_scale, s->act_sum, w, ws, out, B, rows, width};
        g.split_acc = rows <= acc_rows ? s->gemm_acc : nullptr;
        g.residual = residual;
        if (deferred) *deferred = false;
        g.finalize_deferred = g.split_acc ? deferred : nullptr;
        return launch_int4_gemm(g, stream);
    };
    auto aligned16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    const bool defer_x = rmsnorm_quant_reg_fits(H) && aligned16(s->x) && aligned16(s->gemm_acc) &&
                         aligned16(m->s_o) && aligned16(m->s_down) && H % 4 == 0;
    const bool defer_gu = quantize_rows_reg_fits(I) && aligned16(s->gate_up) && aligned16(s->gemm_acc) &&
                          aligned16(m->s_gate_up) && (reinterpret_cast<uintptr_t>(s->x8) & 3) == 0;
    PendingSums pend_x;  // o / down sums pending on x, applied by the next RMSNorm quantisation
    auto norm_quant = [&](const float* gamma) {
        const int r = launch_rmsnorm_quant(s->x, gamma, m->eps, H, B, s->x8, s->act_scale, s->act_sum, stream,
                                           pend_x);
        pend_x = PendingSums{};
        return r;
    };
    batch_embed_kernel<<<B, 256, 0, stream>>>(s->tokens, m->w_embed, m->s_embed, m->vocab, H, s->x);
    H4B_CUDA_TRY(cudaGetLastError());
    for (int l = 0; l < m->layers; ++l) {
        if ((rc = norm_quant(m->norm_in + static_cast<size_t>(l) * H))) return rc;
        if ((rc = gemm(m->w_qkv + static_cast<size_t>(l) * qkv_rows * (H / 2), m->s_qkv + static_cast<size_t>(l) * qkv_rows,
                       s->qkv, qkv_rows, H)))
            return rc;
        if ((rc = batch_attention(m, s, l, stream))) return rc;
        // residual adds in the o / down GEMM epilogues, SwiGLU in the
        // quantisation of its rows (the separate kernels' operations)
        if ((rc = launch_quantize_rows<false>(s->attended, q_size, B, s->x8, s->act_scale, s->act_sum, nullptr,
                                              stream)))
            return rc;
        bool deferred = false;
        const float* s_o = m->s_o + static_cast<size_t>(l) * H;
        if ((rc = gemm(m->w_o + static_cast<size_t>(l) * H * (q_size / 2), s_o, s->x, H, q_size, true,
                       defer_x ? &deferred : nullptr)))
            return rc;
        if (deferred) pend_x = PendingSums{s->gemm_acc, s->act_scale, s_o, H};
        if ((rc = norm_quant(m->norm_post + static_cast<size_t>(l) * H))) return rc;
        const float* s_gu = m->s_gate_up + static_cast<size_t>(l) * 2 * I;
        deferred = false;
        if ((rc = gemm(m->w_gate_up + static_cast<size_t>(l) * 2 * I * (H / 2), s_gu, s->gate_up, 2 * I, H, false,
                       defer_gu ? &deferred : nullptr)))
            return rc;
        const PendingSums pend_gu = deferred ? PendingSums{s->gemm_acc, s->act_scale, s_gu, 2 * I} : PendingSums{};
        if ((rc = launch_quantize_rows<true>(s->gate_up, I, B, s->x8, s->act_scale, s->act_sum, s->act, stream,
                                             pend_gu)))
            return rc;
        const float* s_down = m->s_down + static_cast<size_t>(l) * H;
        deferred = false;
        if ((rc = gemm(m->w_down + static_cast<size_t>(l) * H * (I / 2), s_down, s->x, H, I, true,
                       defer_x ? &deferred : nullptr)))
            return rc;
        if (deferred) pend_x = PendingSums{s->gemm_acc, s->act_scale, s_down, H};  // the next RMSNorm applies it
    }
    if ((rc = norm_quant(m->norm_final))) return rc;
    if ((rc = gemm(m->w_embed, m->s_embed, s->logits, m->vocab, H))) return rc;
    batch_argmax_kernel<<<B, 1024, 0, stream>>>(s->logits, m->vocab, s->next_tokens);
    H4B_CUDA_TRY(cudaGetLastError());
    H4B_CUDA_TRY(cudaMemcpyAsync(s->tokens, s->next_tokens, sizeof(int32_t) * B, cudaMemcpyDeviceToDevice, stream));
    batch_advance_kernel<<<(B + 127) / 128, 128, 0, stream>>>(s->positions, B);
    H4B_CUDA_TRY(cudaGetLastError());
    return 0;
}

}  // namespace h4b

extern "C" int h4b_validate_batch(const h4b_model* model, const h4b_batch_state* state) {
    return h4b::validate_batch(model, state);
}

extern "C" int h4b_batch_attention(const h4b_model* model, const h4b_batch_state* state, int layer, void* stream) {
    int rc = h4b::validate_batch(model, state);
    if (rc) return rc;
    if (layer < 0 || layer >= model->layers) return H4B_EINVAL;
    return h4b::batch_attention(model, state, layer, static_cast<cudaStream_t>(stream));
}

extern "C" int h4b_decode_batch(const h4b_model* model, const h4b_batch_state* state, void* stream) {
    return h4b::decode_batch(model, state, static_cast<cudaStream_t>(stream));
}
