// Batched int4 x int8 product for M > 1 tokens (batched decode, prefill):
//   out[m][n] = float(sum_k w[n][k] * x[m][k]) * act_scale[m] * w_scale[n]
// with w the packed int4 rows (low nibble = even k, codes in [-7, 7]) and x
// each token's int8 activation. The int32 sums are exact, so every row of
// the result equals what the single-token GEMV gives that token.
//
// Tensor-core tiles (mma.sync m16n8k32, u8 x s8 -> s32): the A operand is 16
// weight rows x 32 k, unpacked in registers from the packed bytes as
// u = n ^ 8 = n + 8 (unsigned 1..15), so the product carries 8 * sum_k x[m][k]
// too; the epilogue removes it with the per-token sum the quantiser
// produces. The B operand is 32 k x 8 tokens straight from the int8
// activations. A CTA computes 128 weight rows x 64 tokens; 8 warps own 16
// rows each and loop over the 8 token groups; K advances 64 at a time
// through a 3-stage cp.async pipeline in shared memory (rows padded by 16
// bytes so the fragment loads do not collide on banks).

namespace h4b {

constexpr int kGemmRows = 128;     // weight rows per CTA
constexpr int kGemmTok = 64;       // tokens per CTA
constexpr int kGemmK = 64;         // k per pipeline stage
constexpr int kGemmStages = 3;
constexpr int kGemmWStride = 48;   // bytes per staged weight row (32 + pad)
constexpr int kGemmXStride = 80;   // bytes per staged token row (64 + pad)
constexpr int kGemmStageBytes = kGemmRows * kGemmWStride + kGemmTok * kGemmXStride;

struct GemmArgs {
    const int8_t* x;        // [M][K]
    const float* act_scale; // [M]
    const int32_t* act_sum; // [M]  sum_k x[m][k]
    const uint8_t* w;       // [N][K/2]
    const float* w_scale;   // [N]
    float* out;             // [M][N]
    int M, N, K;
    int32_t* out_i32 = nullptr;  // when set: the exact int32 sums [M][N] instead of `out`
    // tcgen05 split-K (only with a float `out`): when set, [M][N] int32 zeros
    // the K slices are added into (exact, in any order); a finalize kernel
    // applies the epilogue and leaves the buffer zero again.
    int32_t* split_acc = nullptr;
    // with a float `out`: out[m][n] = out[m][n] + value (the residual add,
    // x + proj in that order) instead of out[m][n] = value
    bool residual = false;
    // when set and the K sum is split through split_acc: no finalize kernel;
    // *finalize_deferred says whether the sums were left pending in split_acc
    // (for the consumer to apply, see PendingSums), else it is set false
    bool* finalize_deferred = nullptr;
};

// GEMM results left as exact int32 sums: value[m][n] = float(acc[m][n]) *
// as[m] * ws[n] (the GEMM epilogue's order), which the consumer applies -- and
// then zeroes acc -- instead of a finalize kernel. acc rows are `stride` wide.
struct PendingSums {
    int32_t* acc = nullptr;
    const float* as = nullptr;
    const float* ws = nullptr;
    int stride = 0;
};
__device__ __forceinline__ float pending_value(int sum, float as, float ws) {
    return __fmul_rn(__fmul_rn(static_cast<float>(sum), as), ws);
}

// cp.async with a source size: bytes past src_bytes are zero-filled.
__device__ __forceinline__ void async_copy16_zfill(void* dst, const void* src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void async_wait_group() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Two packed bytes (4 codes, k order lo0 hi0 lo1 hi1) -> 4 unsigned bytes n ^ 8.
__device__ __forceinline__ uint32_t unpack4_u8(uint32_t two_bytes) {
    const uint32_t t = __byte_perm(two_bytes, 0, 0x1100);  // [b0 b0 b1 b1]
    return ((t & 0x000F000Fu) | ((t >> 4) & 0x0F000F00u)) ^ 0x08080808u;
}

__device__ __forceinline__ void mma_u8s8(int d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void gemm_load_stage(const GemmArgs& g, uint8_t* stage, int n0, int m0, int k0) {
    const int tid = threadIdx.x;
    {  // weights: 128 rows x 32 bytes (two 16-byte pieces per row)
        const int row = tid >> 1, piece = tid & 1;
        const uint8_t* src = g.w + static_cast<size_t>(n0 + row) * (g.K / 2) + k0 / 2 + 16 * piece;
        async_copy16_zfill(stage + row * kGemmWStride + 16 * piece, src, 16);
    }
    {  // activations: 64 tokens x 64 bytes (four pieces per token); tokens past M read zeros
        const int tok = tid >> 2, piece = tid & 3;
        const int m = m0 + tok;
        const int8_t* src = g.x + static_cast<size_t>(m < g.M ? m : 0) * g.K + k0 + 16 * piece;
        async_copy16_zfill(stage + kGemmRows * kGemmWStride + tok * kGemmXStride + 16 * piece, src,
                           m < g.M ? 16 : 0);
    }
}

__global__ void __launch_bounds__(256) int4_gemm_kernel(const GemmArgs g) {
    extern __shared__ __align__(128) uint8_t gemm_smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gid = lane >> 2, tig = lane & 3;
    const int n0 = blockIdx.x * kGemmRows, m0 = blockIdx.y * kGemmTok;
    const int steps = g.K / kGemmK;

    int acc[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[j][q] = 0;

#pragma unroll
    for (int s = 0; s < kGemmStages - 1; ++s) {
        if (s < steps) gemm_load_stage(g, gemm_smem + s * kGemmStageBytes, n0, m0, s * kGemmK);
        async_commit();
    }
    for (int step = 0; step < steps; ++step) {
        async_wait_group<kGemmStages - 2>();
        __syncthreads();  // stage `step` is visible; the stage refilled below is no longer read
        const int next = step + kGemmStages - 1;
        if (next < steps) gemm_load_stage(g, gemm_smem + (next % kGemmStages) * kGemmStageBytes, n0, m0, next * kGemmK);
        async_commit();

        const uint8_t* ws = gemm_smem + (step % kGemmStages) * kGemmStageBytes;
        const uint8_t* xs = ws + kGemmRows * kGemmWStride;
        const uint8_t* wrow0 = ws + (16 * warp + gid) * kGemmWStride;
        const uint8_t* wrow8 = wrow0 + 8 * kGemmWStride;
#pragma unroll
        for (int kk = 0; kk < kGemmK; kk += 32) {
            uint32_t a[4];
            a[0] = unpack4_u8(*reinterpret_cast<const uint16_t*>(wrow0 + kk / 2 + 2 * tig));
            a[1] = unpack4_u8(*reinterpret_cast<const uint16_t*>(wrow8 + kk / 2 + 2 * tig));
            a[2] = unpack4_u8(*reinterpret_cast<const uint16_t*>(wrow0 + kk / 2 + 8 + 2 * tig));
            a[3] = unpack4_u8(*reinterpret_cast<const uint16_t*>(wrow8 + kk / 2 + 8 + 2 * tig));
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint8_t* xt = xs + (8 * j + gid) * kGemmXStride + kk + 4 * tig;
                mma_u8s8(acc[j], a, *reinterpret_cast<const uint32_t*>(xt),
                         *reinterpret_cast<const uint32_t*>(xt + 16));
            }
        }
    }
    async_wait_group<0>();

    // epilogue: acc[j] = {(row gid, tok 2t), (row gid, tok 2t+1), (row gid+8, tok 2t), (row gid+8, tok 2t+1)}
    const int r0 = n0 + 16 * warp + gid;
    const float ws0 = g.w_scale[r0], ws8 = g.w_scale[r0 + 8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
        for (int c = 0; c < 2; ++c) {
            const int m = m0 + 8 * j + 2 * tig + c;
            if (m >= g.M) continue;
            const int bias = -8 * g.act_sum[m];
            if (g.out_i32) {
                int32_t* irow = g.out_i32 + static_cast<size_t>(m) * g.N;
                irow[r0] = acc[j][c] + bias;
                irow[r0 + 8] = acc[j][2 + c] + bias;
                continue;
            }
            const float as = g.act_scale[m];
            float* orow = g.out + static_cast<size_t>(m) * g.N;
            const float v0 = __fmul_rn(__fmul_rn(static_cast<float>(acc[j][c] + bias), as), ws0);
            const float v8 = __fmul_rn(__fmul_rn(static_cast<float>(acc[j][2 + c] + bias), as), ws8);
            orow[r0] = g.residual ? __fadd_rn(orow[r0], v0) : v0;
            orow[r0 + 8] = g.residual ? __fadd_rn(orow[r0 + 8], v8) : v8;
        }
    }
}

// Per-token quantisation of M rows (the quantize_activation contract per row)
// plus each row's int8 sum: one CTA per row.
// With `given_max`, row r is quantised with the absmax given_max[r] (a
// maximum taken over more values than this row holds, e.g. over the ranks of
// a tensor-parallel group) instead of its own.
__global__ void __launch_bounds__(256) quantize_rows_kernel(const float* v, int K, int8_t* q, float* scales,
                                                            int32_t* sums, const float* given_max = nullptr) {
    __shared__ float red[8];
    __shared__ int ired[8];
    const float* row = v + static_cast<size_t>(blockIdx.x) * K;
    float m;
    if (given_max) {
        m = given_max[blockIdx.x];
    } else {
        float mx = 0.f;
        for (int i = threadIdx.x; i < K; i += blockDim.x) mx = fmaxf(mx, fabsf(row[i]));
        mx = warp_max(mx);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
        __syncthreads();
        m = red[0];
        for (int w = 1; w < 8; ++w) m = fmaxf(m, red[w]);
    }
    const float qs = quant_multiplier(m);
    int s = 0;
    int8_t* qrow = q + static_cast<size_t>(blockIdx.x) * K;
    for (int i = threadIdx.x; i < K; i += blockDim.x) {
        const int qi = quantize_one(row[i], qs);
        qrow[i] = static_cast<int8_t>(qi);
        s += qi;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) ired[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        int t = 0;
        for (int w = 0; w < 8; ++w) t += ired[w];
        sums[blockIdx.x] = t;
        scales[blockIdx.x] = dequant_scale(m);
    }
}

// quantize_rows_kernel's result, bit for bit, with the row read once into
// registers (float4 loads, kGroups groups of 4 per thread). With kSwiglu the
// row is act = silu(gate) * up from the interleaved gate/up row
// (batch_swiglu_kernel's arithmetic; [gate x4][up x4] per group), and act
// itself is never stored. The maximum and the code sum are order-free.
template <int kThreads, int kGroups, bool kSwiglu>
__global__ void __launch_bounds__(kThreads) quantize_rows_reg_kernel(const float* v, int K, int8_t* q,
                                                                    float* scales, int32_t* sums, PendingSums pend) {
    __shared__ float red[kThreads / 32];
    __shared__ int ired[kThreads / 32];
    const int groups = K / 4;
    const float4* row = reinterpret_cast<const float4*>(v + static_cast<size_t>(blockIdx.x) * (kSwiglu ? 2 : 1) * K);
    // pending GEMM sums instead of v (SwiGLU rows only): read before this
    // row's scale is overwritten below (after the barriers)
    int4* prow = pend.acc ? reinterpret_cast<int4*>(pend.acc + static_cast<size_t>(blockIdx.x) * pend.stride) : nullptr;
    const float pas = pend.acc ? pend.as[blockIdx.x] : 0.f;
    const float4* pws = reinterpret_cast<const float4*>(pend.ws);
    float4 a[kGroups];
    float mx = 0.f;
#pragma unroll
    for (int k = 0; k < kGroups; ++k) {
        const int gi = threadIdx.x + k * kThreads;
        a[k] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (gi < groups) {
            if constexpr (kSwiglu) {
                float4 g, u;
                if (prow) {
                    const int4 sg = prow[2 * gi], su = prow[2 * gi + 1];
                    const float4 wg = pws[2 * gi], wu = pws[2 * gi + 1];
                    g = make_float4(pending_value(sg.x, pas, wg.x), pending_value(sg.y, pas, wg.y),
                                    pending_value(sg.z, pas, wg.z), pending_value(sg.w, pas, wg.w));
                    u = make_float4(pending_value(su.x, pas, wu.x), pending_value(su.y, pas, wu.y),
                                    pending_value(su.z, pas, wu.z), pending_value(su.w, pas, wu.w));
                    prow[2 * gi] = make_int4(0, 0, 0, 0);
                    prow[2 * gi + 1] = make_int4(0, 0, 0, 0);
                } else {
                    g = row[2 * gi];
                    u = row[2 * gi + 1];
                }
                a[k] = make_float4(swiglu_one(g.x, u.x), swiglu_one(g.y, u.y), swiglu_one(g.z, u.z),
                                   swiglu_one(g.w, u.w));
            } else {
                a[k] = row[gi];
            }
            mx = fmaxf(fmaxf(mx, fabsf(a[k].x)), fmaxf(fabsf(a[k].y), fmaxf(fabsf(a[k].z), fabsf(a[k].w))));
        }
    }
    mx = warp_max(mx);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    float m = red[0];
#pragma unroll
    for (int w = 1; w < kThreads / 32; ++w) m = fmaxf(m, red[w]);
    const float qs = quant_multiplier(m);
    int s = 0;
    uint32_t* qrow = reinterpret_cast<uint32_t*>(q + static_cast<size_t>(blockIdx.x) * K);
#pragma unroll
    for (int k = 0; k < kGroups; ++k) {
        const int gi = threadIdx.x + k * kThreads;
        if (gi < groups) {
            const int c0 = quantize_one(a[k].x, qs), c1 = quantize_one(a[k].y, qs);
            const int c2 = quantize_one(a[k].z, qs), c3 = quantize_one(a[k].w, qs);
            qrow[gi] = (static_cast<uint32_t>(c0) & 0xFFu) | ((static_cast<uint32_t>(c1) & 0xFFu) << 8) |
                       ((static_cast<uint32_t>(c2) & 0xFFu) << 16) | (static_cast<uint32_t>(c3) << 24);
            s += c0 + c1 + c2 + c3;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) ired[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        int t = 0;
        for (int w = 0; w < kThreads / 32; ++w) t += ired[w];
        sums[blockIdx.x] = t;
        scales[blockIdx.x] = dequant_scale(m);
    }
}

constexpr int kQuantThreads = 512, kQuantMaxGroups = 8;

__global__ void batch_swiglu_kernel(const float* gate_up, int I, int B, float* act);  // batch.cu

template <bool kSwiglu, int G>
void launch_quantize_reg(const float* v, int K, int rows, int8_t* q, float* scales, int32_t* sums,
                         cudaStream_t stream, PendingSums pend) {
    quantize_rows_reg_kernel<kQuantThreads, G, kSwiglu><<<rows, kQuantThreads, 0, stream>>>(v, K, q, scales, sums,
                                                                                           pend);
}

// Whether launch_quantize_rows takes its register kernel (the only one that
// applies pending GEMM sums) for rows of K values.
inline bool quantize_rows_reg_fits(int K) {
    return K % 4 == 0 && (K / 4 + kQuantThreads - 1) / kQuantThreads <= kQuantMaxGroups;
}

// Per-row quantisation of `rows` rows of K values (kSwiglu: of the SwiGLU of
// `rows` interleaved gate/up rows of 2K values) into q / scales / sums; the
// register kernel when a row fits, else the general kernels (kSwiglu then
// needs `act`, [rows][K], for the intermediate values).
template <bool kSwiglu>
int launch_quantize_rows(const float* v, int K, int rows, int8_t* q, float* scales, int32_t* sums, float* act,
                         cudaStream_t stream, PendingSums pend = {}) {
    const int per = (K / 4 + kQuantThreads - 1) / kQuantThreads;
    if (pend.acc && (!kSwiglu || !quantize_rows_reg_fits(K) || pend.stride % 4 != 0 ||
                     ((reinterpret_cast<uintptr_t>(pend.acc) | reinterpret_cast<uintptr_t>(pend.ws)) & 15) != 0))
        return H4B_EUNSUPPORTED;
    if (quantize_rows_reg_fits(K) && (reinterpret_cast<uintptr_t>(v) & 15) == 0 &&
        (reinterpret_cast<uintptr_t>(q) & 3) == 0) {
        switch (per) {
            case 0:
            case 1: launch_quantize_reg<kSwiglu, 1>(v, K, rows, q, scales, sums, stream, pend); break;
            case 2: launch_quantize_reg<kSwiglu, 2>(v, K, rows, q, scales, sums, stream, pend); break;
            case 3: launch_quantize_reg<kSwiglu, 3>(v, K, rows, q, scales, sums, stream, pend); break;
            case 4: launch_quantize_reg<kSwiglu, 4>(v, K, rows, q, scales, sums, stream, pend); break;
            case 5: launch_quantize_reg<kSwiglu, 5>(v, K, rows, q, scales, sums, stream, pend); break;
            case 6: launch_quantize_reg<kSwiglu, 6>(v, K, rows, q, scales, sums, stream, pend); break;
            default: launch_quantize_reg<kSwiglu, 8>(v, K, rows, q, scales, sums, stream, pend); break;
        }
        H4B_CUDA_TRY(cudaGetLastError());
        return 0;
    }
    if (pend.acc) return H4B_EUNSUPPORTED;
    const float* src = v;
    if constexpr (kSwiglu) {
        if (!act) return H4B_EUNSUPPORTED;
        const long long n = static_cast<long long>(rows) * K;
        batch_swiglu_kernel<<<static_cast<int>((n + 255) / 256), 256, 0, stream>>>(v, K, rows, act);
        src = act;
    }
    quantize_rows_kernel<<<rows, 256, 0, stream>>>(src, K, q, scales, sums);
    H4B_CUDA_TRY(cudaGetLastError());
    return 0;
}

int launch_int4_gemm_mma(const GemmArgs& g, cudaStream_t stream) {
    if (g.M < 1 || g.N < 1 || g.K < 1) return H4B_EINVAL;
    if (g.N % kGemmRows || g.K % kGemmK) return H4B_EUNSUPPORTED;
    const dim3 grid(g.N / kGemmRows, (g.M + kGemmTok - 1) / kGemmTok);
    int4_gemm_kernel<<<grid, 256, kGemmStages * kGemmStageBytes, stream>>>(g);
    H4B_CUDA_TRY(cudaGetLastError());
    return 0;
}

}  // namespace h4b
