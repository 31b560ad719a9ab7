// Stochastic token sampling on the device (reference semantics:
// inference_runtime.sample_numpy, inference_runtime.py:144-163, and
// cpu_lightspark.sample_logits, cpu_lightspark.py:700-726).
//
//   values = logits; values[seen] = v > 0 ? v / penalty : v * penalty
//   temperature <= 0.01 -> argmax(values) (first maximum)
//   values /= T; ids = top-k(values) sorted descending
//   p = exp(v_ids - max) / sum; p[(cumsum(p) - p) >= top_p] = 0; p /= sum(p)
//   token = ids[searchsorted(cumsum_f64(p) / last, u, side = right)]
//
// numpy's Generator.choice(ids, p) draws u = random() and performs exactly
// that float64 CDF search, so a host that draws u from the same generator
// gets the same token as the reference (up to last-ulp differences of exp).
// Sums over the k probabilities follow numpy's float32 pairwise summation
// (8 running partials, then ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)), then the
// remainder), cumulative sums are sequential.
//
// Pass 1: blocks of 1024 threads sort 2048 scaled values each (bitonic, in
// shared memory) and keep their top k. Pass 2: one block sorts the
// candidates and thread 0 does the k-element tail in numpy's order.

namespace h4b {

constexpr int kSampleMaxK = 64;
constexpr int kSampleChunk = 2048;      // values sorted per pass-1 block
constexpr int kSampleMaxCand = 8192;    // pass-2 sort size (candidates padded)

// (value, index) ordered by value descending, then index ascending.
__device__ __forceinline__ bool sample_before(float va, int ia, float vb, int ib) {
    return va > vb || (va == vb && ia < ib);
}

// Bitonic sort of n (a power of two) pairs in shared memory, descending.
__device__ void sample_bitonic(float* v, int* ix, int n) {
    for (int size = 2; size <= n; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int t = threadIdx.x; t < (n >> 1); t += blockDim.x) {
                const int pos = 2 * t - (t & (stride - 1));
                const int other = pos + stride;
                const bool desc = (pos & size) == 0;
                const bool first_wins = sample_before(v[pos], ix[pos], v[other], ix[other]);
                if (desc != first_wins) {
                    const float tv = v[pos];
                    v[pos] = v[other];
                    v[other] = tv;
                    const int ti = ix[pos];
                    ix[pos] = ix[other];
                    ix[other] = ti;
                }
            }
            __syncthreads();
        }
    }
}

__global__ void sample_penalty_kernel(float* logits, const int32_t* ids, int n, int vocab, float penalty) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int id = ids[i];
    if (id < 0 || id >= vocab) return;
    const float v = logits[id];
    logits[id] = v > 0.f ? __fdiv_rn(v, penalty) : __fmul_rn(v, penalty);
}

__global__ void __launch_bounds__(1024) sample_topk_block_kernel(const float* logits, int vocab, float temperature,
                                                                 int k, float* cand_v, int* cand_i) {
    __shared__ float v[kSampleChunk];
    __shared__ int ix[kSampleChunk];
    const int base = blockIdx.x * kSampleChunk;
    for (int t = threadIdx.x; t < kSampleChunk; t += blockDim.x) {
        const int i = base + t;
        v[t] = i < vocab ? __fdiv_rn(logits[i], temperature) : -INFINITY;
        ix[t] = i < vocab ? i : 0x7fffffff;
    }
    __syncthreads();
    sample_bitonic(v, ix, kSampleChunk);
    for (int j = threadIdx.x; j < k; j += blockDim.x) {
        cand_v[blockIdx.x * k + j] = v[j];
        cand_i[blockIdx.x * k + j] = ix[j];
    }
}

// numpy float32 pairwise sum of n <= 128 contiguous values.
__device__ float numpy_sum_f32(const float* a, int n) {
    if (n < 8) {
        float r = 0.f;
        for (int i = 0; i < n; ++i) r = __fadd_rn(r, a[i]);
        return r;
    }
    float r[8];
    for (int j = 0; j < 8; ++j) r[j] = a[j];
    int i = 8;
    for (; i < n - (n % 8); i += 8)
        for (int j = 0; j < 8; ++j) r[j] = __fadd_rn(r[j], a[i + j]);
    float res = __fadd_rn(__fadd_rn(__fadd_rn(r[0], r[1]), __fadd_rn(r[2], r[3])),
                          __fadd_rn(__fadd_rn(r[4], r[5]), __fadd_rn(r[6], r[7])));
    for (; i < n; ++i) res = __fadd_rn(res, a[i]);
    return res;
}

__global__ void __launch_bounds__(1024) sample_final_kernel(const float* cand_v, const int* cand_i, int n_cand, int k,
                                                            float top_p, double uniform, int32_t* token_out,
                                                            int32_t* ids_out, float* probs_out) {
    extern __shared__ __align__(16) uint8_t sample_smem[];
    int n = 1;
    while (n < n_cand) n <<= 1;
    float* v = reinterpret_cast<float*>(sample_smem);
    int* ix = reinterpret_cast<int*>(v + n);
    for (int t = threadIdx.x; t < n; t += blockDim.x) {
        v[t] = t < n_cand ? cand_v[t] : -INFINITY;
        ix[t] = t < n_cand ? cand_i[t] : 0x7fffffff;
    }
    __syncthreads();
    sample_bitonic(v, ix, n);
    if (threadIdx.x != 0) return;
    float p[kSampleMaxK];
    const float mx = v[0];
    for (int j = 0; j < k; ++j) p[j] = expf(__fsub_rn(v[j], mx));
    float sum = numpy_sum_f32(p, k);
    for (int j = 0; j < k; ++j) p[j] = __fdiv_rn(p[j], sum);
    if (top_p < 1.0f) {
        bool drop[kSampleMaxK];
        float c = 0.f;
        for (int j = 0; j < k; ++j) {
            c = j == 0 ? p[0] : __fadd_rn(c, p[j]);
            drop[j] = __fsub_rn(c, p[j]) >= top_p;
        }
        for (int j = 0; j < k; ++j)
            if (drop[j]) p[j] = 0.f;
        sum = numpy_sum_f32(p, k);
        for (int j = 0; j < k; ++j) p[j] = __fdiv_rn(p[j], sum);
    }
    double cdf[kSampleMaxK];
    double acc = 0.0;
    for (int j = 0; j < k; ++j) {
        acc = __dadd_rn(acc, static_cast<double>(p[j]));
        cdf[j] = acc;
    }
    int pick = k - 1;
    for (int j = 0; j < k; ++j) {
        if (__ddiv_rn(cdf[j], cdf[k - 1]) > uniform) {
            pick = j;
            break;
        }
    }
    *token_out = ix[pick];
    if (ids_out)
        for (int j = 0; j < k; ++j) ids_out[j] = ix[j];
    if (probs_out)
        for (int j = 0; j < k; ++j) probs_out[j] = p[j];
}

size_t sample_scratch_bytes(int vocab, int top_k) {
    const int blocks = (vocab + kSampleChunk - 1) / kSampleChunk;
    return static_cast<size_t>(blocks) * top_k * (sizeof(float) + sizeof(int));
}

int sample_tokens(float* logits, int vocab, const int32_t* generated, int n_generated, float temperature, int top_k,
                  float top_p, float penalty, double uniform, int32_t* token_out, int32_t* ids_out, float* probs_out,
                  void* scratch, cudaStream_t stream) {
    if (!logits || !token_out || vocab < 1 || n_generated < 0 || (n_generated > 0 && !generated)) return H4B_EINVAL;
    if (!(uniform >= 0.0 && uniform < 1.0) || !(penalty > 0.f)) return H4B_EINVAL;
    if (n_generated > 0 && penalty != 1.0f) {
        sample_penalty_kernel<<<(n_generated + 255) / 256, 256, 0, stream>>>(logits, generated, n_generated, vocab,
                                                                            penalty);
        H4B_CUDA_TRY(cudaGetLastError());
    }
    if (temperature <= 0.01f) {  // greedy on the penalised values
        argmax_kernel<<<1, 1024, 0, stream>>>(logits, vocab, token_out);
        H4B_CUDA_TRY(cudaGetLastError());
        return 0;
    }
    const int k = top_k > 0 ? std::min(top_k, vocab) : std::min(50, vocab);
    if (k > kSampleMaxK) return H4B_EUNSUPPORTED;
    if (!scratch) return H4B_EINVAL;
    const int blocks = (vocab + kSampleChunk - 1) / kSampleChunk;
    const int n_cand = blocks * k;
    if (n_cand > kSampleMaxCand) return H4B_ETOOBIG;
    float* cand_v = static_cast<float*>(scratch);
    int* cand_i = reinterpret_cast<int*>(cand_v + n_cand);
    sample_topk_block_kernel<<<blocks, 1024, 0, stream>>>(logits, vocab, temperature, k, cand_v, cand_i);
    H4B_CUDA_TRY(cudaGetLastError());
    int n = 1;
    while (n < n_cand) n <<= 1;
    sample_final_kernel<<<1, 1024, n * 8, stream>>>(cand_v, cand_i, n_cand, k, top_p, uniform, token_out, ids_out,
                                                     probs_out);
    H4B_CUDA_TRY(cudaGetLastError());
    return 0;
}

int prepare_sampling() {
    return cudaFuncSetAttribute(sample_final_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSampleMaxCand * 8);
}

}  // namespace h4b

extern "C" long long h4b_sample_scratch_bytes(int vocab, int top_k) {
    if (vocab < 1) return H4B_EINVAL;
    const int k = top_k > 0 ? std::min(top_k, vocab) : std::min(50, vocab);
    if (k > h4b::kSampleMaxK) return H4B_EUNSUPPORTED;
    return static_cast<long long>(h4b::sample_scratch_bytes(vocab, k));
}

extern "C" int h4b_sample(float* logits, int vocab, const int32_t* generated, int n_generated, float temperature,
                          int top_k, float top_p, float repetition_penalty, double uniform, int32_t* token_out,
                          int32_t* topk_ids_out, float* topk_probs_out, void* scratch, void* stream) {
    return h4b::sample_tokens(logits, vocab, generated, n_generated, temperature, top_k, top_p, repetition_penalty,
                              uniform, token_out, topk_ids_out, topk_probs_out, scratch,
                              static_cast<cudaStream_t>(stream));
}
