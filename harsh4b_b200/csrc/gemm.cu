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
};

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
            orow[r0] = __fmul_rn(__fmul_rn(static_cast<float>(acc[j][c] + bias), as), ws0);
            orow[r0 + 8] = __fmul_rn(__fmul_rn(static_cast<float>(acc[j][2 + c] + bias), as), ws8);
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

int launch_int4_gemm_mma(const GemmArgs& g, cudaStream_t stream) {
    if (g.M < 1 || g.N < 1 || g.K < 1) return H4B_EINVAL;
    if (g.N % kGemmRows || g.K % kGemmK) return H4B_EUNSUPPORTED;
    const dim3 grid(g.N / kGemmRows, (g.M + kGemmTok - 1) / kGemmTok);
    int4_gemm_kernel<<<grid, 256, kGemmStages * kGemmStageBytes, stream>>>(g);
    H4B_CUDA_TRY(cudaGetLastError());
    return 0;
}

}  // namespace h4b
