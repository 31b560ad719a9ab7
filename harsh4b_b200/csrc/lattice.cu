// LATTICE -> row-int4 conversion on the GPU: the one-time step that builds
// the packed cache from the LATTICE checkpoint (the reference does it on the
// CPU in cpu_lightspark._convert_projection, cpu_lightspark.py:149-201, with
// MLX/lattice_model.expand_t1, :160-185, and _convert_embedding,
// cpu_lightspark.py:204-229).
//
// Projection, per row r and column c (b = c / blocksize, m = mode id):
//   w[c] = mu[m][r][b] + a0[m][r][b] * trit(T0[c])
//          + sum over i of [m == o2[i]] * a1[i][r][b] * trit(T1[c])
// (fp32, added in that order; trit(0..3) = 0, +1, -1, 0), where T1 holds a
// code only for the columns with m < 2, stored compactly in row-major order
// across the whole matrix. Then the KOTMS rotation is absorbed per row,
// W_r (dim_l x dim_r) -> L^T W_r R^T, and the row is quantised:
//   scale = max(max|w|, 1e-8) / 7,  code = clip(rint(w / scale), -7, 7),
// packed two per byte (low nibble = even column).
//
// The rotation is accumulated in fp64 and rounded once to fp32 (the
// reference uses an fp32 BLAS product whose summation order is the
// library's), so codes can differ from the reference's by one where w/scale
// lies within a few ulp of a rounding boundary; everything else is exact.
// The embedding / dense-row conversion has no product and is bit-exact.

namespace h4b {

__device__ __forceinline__ int lat_code(const uint8_t* row, int j) { return (row[j >> 2] >> ((j & 3) * 2)) & 3; }
__device__ __forceinline__ float lat_trit(int code) { return code == 1 ? 1.0f : (code == 2 ? -1.0f : 0.0f); }

// counts[r] = columns of row r whose mode id is 0 or 1 (the ones with a T1
// code). A 2-bit code is < 2 exactly when its high bit is clear.
__global__ void lattice_t1_counts_kernel(const uint8_t* maskid, int rows, int width, int row_bytes,
                                         long long* counts) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    for (int r = warp; r < rows; r += nwarps) {
        const uint8_t* row = maskid + static_cast<size_t>(r) * row_bytes;
        int n = 0;
        for (int j = lane; j < row_bytes; j += 32) {
            const int valid = min(4, width - 4 * j);  // columns held by this byte
            const uint32_t hi = (row[j] >> 1) & 0x55u & ((1u << (2 * valid)) - 1u);
            n += valid - __popc(hi);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) n += __shfl_xor_sync(0xffffffffu, n, o);
        if (lane == 0) counts[r] = n;
    }
}

// starts[r] = sum of counts[0..r), starts[rows] = total. One CTA.
constexpr int kScanThreads = 1024;
__global__ void __launch_bounds__(kScanThreads) lattice_scan_kernel(const long long* counts, int rows,
                                                                    long long* starts) {
    __shared__ long long part[kScanThreads];
    const int t = threadIdx.x;
    const int chunk = (rows + kScanThreads - 1) / kScanThreads;
    const int r0 = min(rows, t * chunk), r1 = min(rows, r0 + chunk);
    long long s = 0;
    for (int r = r0; r < r1; ++r) s += counts[r];
    part[t] = s;
    __syncthreads();
    for (int off = 1; off < kScanThreads; off <<= 1) {  // inclusive Hillis-Steele scan
        const long long v = t >= off ? part[t - off] : 0;
        __syncthreads();
        part[t] += v;
        __syncthreads();
    }
    long long run = part[t] - s;  // exclusive prefix of this thread's chunk
    for (int r = r0; r < r1; ++r) {
        starts[r] = run;
        run += counts[r];
    }
    if (t == kScanThreads - 1) starts[rows] = part[t];
}

struct LatArgs {
    h4b_lattice_projection p;
    const long long* starts;
    uint8_t* packed;
    float* scales;
    int* error;  // device word: set to 1 if a T1 index runs past the compact codes
};

constexpr int kLatThreads = 256;

template <typename P>
__device__ __forceinline__ float lat_param(const void* base, size_t i) {
    return static_cast<float>(static_cast<const P*>(base)[i]);
}

__device__ __forceinline__ float lat_block_max(float v, float* red) {
    v = warp_max(v);
    const int warp = threadIdx.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[warp] = v;
    __syncthreads();
    float m = red[0];
    for (int w = 1; w < (kLatThreads >> 5); ++w) m = fmaxf(m, red[w]);
    return m;
}

// One CTA per row (grid-stride). Shared memory: the row's fp32 weights
// [width], the fp64 product W R^T [width], and, with STAGE, R and L.
template <typename P, bool STAGE>
__global__ void __launch_bounds__(kLatThreads) lattice_convert_kernel(const LatArgs a) {
    extern __shared__ __align__(16) uint8_t lat_smem[];
    const h4b_lattice_projection& p = a.p;
    const int width = p.width, dl = p.dim_l, dr = p.dim_r;
    double* prod = reinterpret_cast<double*>(lat_smem);           // [dl][dr]
    float* w = reinterpret_cast<float*>(prod + width);             // [width]
    float* rs = w + width;                                         // [dr][dr] when STAGE
    float* ls = rs + (STAGE ? dr * dr : 0);                        // [dl][dl] when STAGE
    __shared__ long long scan[kLatThreads];
    __shared__ float red[kLatThreads / 32];
    const float* R = STAGE ? rs : p.right;
    const float* L = STAGE ? ls : p.left;
    const int tid = threadIdx.x;
    const int row_bytes = (width + 3) >> 2;
    if (STAGE) {
        for (int i = tid; i < dr * dr; i += kLatThreads) rs[i] = p.right[i];
        for (int i = tid; i < dl * dl; i += kLatThreads) ls[i] = p.left[i];
    }
    const int chunk = (width + kLatThreads - 1) / kLatThreads;  // contiguous columns per thread
    const int c0 = min(width, tid * chunk), c1 = min(width, c0 + chunk);
    for (int r = blockIdx.x; r < p.rows; r += gridDim.x) {
        const uint8_t* mrow = p.maskid + static_cast<size_t>(r) * row_bytes;
        const uint8_t* trow = p.t0 + static_cast<size_t>(r) * row_bytes;
        // In-row position of each T1 code: exclusive scan of this thread's count.
        long long mine = 0;
        for (int c = c0; c < c1; ++c) mine += lat_code(mrow, c) < 2;
        __syncthreads();  // the previous row is done with scan[], prod[], w[]
        scan[tid] = mine;
        __syncthreads();
        for (int off = 1; off < kLatThreads; off <<= 1) {
            const long long v = tid >= off ? scan[tid - off] : 0;
            __syncthreads();
            scan[tid] += v;
            __syncthreads();
        }
        long long idx = a.starts[r] + scan[tid] - mine;
        bool bad = false;
        for (int c = c0; c < c1; ++c) {
            const int m = lat_code(mrow, c);
            const int b = c / p.blocksize;
            int code1 = 0;
            if (m < 2) {
                if (idx < p.n_t1 && (idx >> 2) < p.t1c_bytes) code1 = (p.t1c[idx >> 2] >> ((idx & 3) * 2)) & 3;
                else bad = true;
                ++idx;
            }
            const size_t mi = (static_cast<size_t>(m) * p.rows + r) * p.nblocks + b;
            float v = lat_param<P>(p.mu, mi);
            v = __fadd_rn(v, __fmul_rn(lat_param<P>(p.a0, mi), lat_trit(lat_code(trow, c))));
            for (int i = 0; i < p.n_o2; ++i) {
                const float term = m == p.o2_idx[i]
                    ? __fmul_rn(lat_param<P>(p.a1, (static_cast<size_t>(i) * p.rows + r) * p.nblocks + b),
                                lat_trit(code1))
                    : 0.0f;
                v = __fadd_rn(v, term);
            }
            w[c] = v;
        }
        if (bad) atomicExch(a.error, 1);
        __syncthreads();
        // prod = W R^T (fp64): prod[i][j] = sum_b W[i][b] R[j][b]
        for (int e = tid; e < width; e += kLatThreads) {
            const int i = e / dr, j = e - i * dr;
            const float* wi = w + i * dr;
            const float* rj = R + static_cast<size_t>(j) * dr;
            double s = 0.0;
            for (int b = 0; b < dr; ++b) s = fma(static_cast<double>(wi[b]), static_cast<double>(rj[b]), s);
            prod[e] = s;
        }
        __syncthreads();
        // out = L^T prod, rounded once to fp32, into w
        float amax = 0.0f;
        for (int e = tid; e < width; e += kLatThreads) {
            const int i = e / dr, j = e - i * dr;
            double s = 0.0;
            for (int k = 0; k < dl; ++k)
                s = fma(static_cast<double>(L[static_cast<size_t>(k) * dl + i]), prod[k * dr + j], s);
            const float v = static_cast<float>(s);
            w[e] = v;
            amax = fmaxf(amax, fabsf(v));
        }
        amax = lat_block_max(amax, red);  // its barriers also publish w[]
        const float scale = __fdiv_rn(fmaxf(amax, 1e-8f), 7.0f);
        uint8_t* out = a.packed + static_cast<size_t>(r) * (width >> 1);
        for (int j = tid; j < (width >> 1); j += kLatThreads) {
            const float lo = fminf(7.0f, fmaxf(-7.0f, rintf(__fdiv_rn(w[2 * j], scale))));
            const float hi = fminf(7.0f, fmaxf(-7.0f, rintf(__fdiv_rn(w[2 * j + 1], scale))));
            out[j] = static_cast<uint8_t>((static_cast<int>(lo) & 15) | ((static_cast<int>(hi) & 15) << 4));
        }
        if (tid == 0) a.scales[r] = scale;
    }
}

// Dense rows -> row int4 (cpu_lightspark.py:204-229): one warp per row.
template <typename S>
__global__ void rows_to_int4_kernel(const S* src, int rows, int width, uint8_t* packed, float* scales) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    for (int r = warp; r < rows; r += nwarps) {
        const S* row = src + static_cast<size_t>(r) * width;
        float amax = 0.0f;
        for (int c = lane; c < width; c += 32) amax = fmaxf(amax, fabsf(static_cast<float>(row[c])));
        amax = warp_max(amax);
        const float scale = __fdiv_rn(fmaxf(amax, 1e-8f), 7.0f);
        uint8_t* out = packed + static_cast<size_t>(r) * (width >> 1);
        for (int j = lane; j < (width >> 1); j += 32) {
            const float lo = fminf(7.0f, fmaxf(-7.0f, rintf(__fdiv_rn(static_cast<float>(row[2 * j]), scale))));
            const float hi = fminf(7.0f, fmaxf(-7.0f, rintf(__fdiv_rn(static_cast<float>(row[2 * j + 1]), scale))));
            out[j] = static_cast<uint8_t>((static_cast<int>(lo) & 15) | ((static_cast<int>(hi) & 15) << 4));
        }
        if (lane == 0) scales[r] = scale;
    }
}

static size_t lat_smem_bytes(int width, int dl, int dr, bool stage) {
    size_t bytes = static_cast<size_t>(width) * (sizeof(double) + sizeof(float));
    if (stage) bytes += (static_cast<size_t>(dr) * dr + static_cast<size_t>(dl) * dl) * sizeof(float);
    return bytes;
}

template <typename P, bool STAGE>
static int launch_lattice(const LatArgs& a, size_t smem, cudaStream_t stream) {
    // Per-device opt-in above the 48 KB default, recording only a success.
    static std::atomic<bool> opted_in[kMaxDevices];
    int dev = 0;
    H4B_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return H4B_EUNSUPPORTED;
    if (!opted_in[dev].load(std::memory_order_acquire)) {
        H4B_CUDA_TRY(cudaFuncSetAttribute(lattice_convert_kernel<P, STAGE>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        opted_in[dev].store(true, std::memory_order_release);
    }
    const int grid = std::max(1, std::min(a.p.rows, sm_count()));
    lattice_convert_kernel<P, STAGE><<<grid, kLatThreads, smem, stream>>>(a);
    H4B_CUDA_TRY(cudaGetLastError());
    return 0;
}

}  // namespace h4b

extern "C" long long h4b_lattice_scratch_bytes(int rows) {
    if (rows < 1) return H4B_EINVAL;
    return (2ll * rows + 1) * static_cast<long long>(sizeof(long long)) + 16;
}

extern "C" int h4b_lattice_to_int4(const h4b_lattice_projection* p, uint8_t* packed, float* scales, void* scratch,
                                   int* host_error, void* stream) {
    using namespace h4b;
    if (!p || !packed || !scales || !scratch || !host_error) return H4B_EINVAL;
    if (!p->maskid || !p->t0 || !p->mu || !p->a0 || !p->left || !p->right) return H4B_EINVAL;
    if (p->rows < 1 || p->width < 2 || (p->width & 1) || p->blocksize < 1 || p->dim_l < 1 || p->dim_r < 1)
        return H4B_EINVAL;
    if (static_cast<long long>(p->dim_l) * p->dim_r != p->width) return H4B_EINVAL;
    if (p->nblocks != (p->width + p->blocksize - 1) / p->blocksize) return H4B_EINVAL;
    if (p->n_o2 < 0 || p->n_o2 > 4 || (p->n_o2 > 0 && !p->a1) || p->n_t1 < 0 || p->t1c_bytes < 0) return H4B_EINVAL;
    if (p->n_t1 > 0 && !p->t1c) return H4B_EINVAL;
    for (int i = 0; i < p->n_o2; ++i)
        if (p->o2_idx[i] < 0 || p->o2_idx[i] > 3) return H4B_EINVAL;
    if (p->param_dtype != 0 && p->param_dtype != 1) return H4B_EINVAL;
    const size_t unstaged = lat_smem_bytes(p->width, p->dim_l, p->dim_r, false);
    if (unstaged > 200 * 1024) return H4B_EUNSUPPORTED;
    if (reinterpret_cast<uintptr_t>(scratch) & 15) return H4B_EINVAL;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    long long* counts = static_cast<long long*>(scratch);
    long long* starts = counts + p->rows;
    int* error = reinterpret_cast<int*>(starts + p->rows + 1);
    H4B_CUDA_TRY(cudaMemsetAsync(error, 0, sizeof(int), s));
    const int row_bytes = (p->width + 3) >> 2;
    lattice_t1_counts_kernel<<<std::max(1, std::min((p->rows + 7) / 8, 4 * sm_count())), 256, 0, s>>>(
        p->maskid, p->rows, p->width, row_bytes, counts);
    H4B_CUDA_TRY(cudaGetLastError());
    lattice_scan_kernel<<<1, kScanThreads, 0, s>>>(counts, p->rows, starts);
    H4B_CUDA_TRY(cudaGetLastError());
    // expand_t1's consistency check (MLX/lattice_model.py:178-183): the mask
    // must select exactly n_T1 codes, all inside the compact buffer.
    long long total = -1;
    H4B_CUDA_TRY(cudaMemcpyAsync(&total, starts + p->rows, sizeof(long long), cudaMemcpyDeviceToHost, s));
    H4B_CUDA_TRY(cudaStreamSynchronize(s));
    if (total != p->n_t1 || (total + 3) / 4 > p->t1c_bytes) {
        *host_error = 1;
        return H4B_EINVAL;
    }
    LatArgs a{*p, starts, packed, scales, error};
    const size_t staged = lat_smem_bytes(p->width, p->dim_l, p->dim_r, true);
    const bool stage = staged <= 200 * 1024;
    int rc;
    if (p->param_dtype == 1)
        rc = stage ? launch_lattice<__half, true>(a, staged, s) : launch_lattice<__half, false>(a, unstaged, s);
    else
        rc = stage ? launch_lattice<float, true>(a, staged, s) : launch_lattice<float, false>(a, unstaged, s);
    if (rc) return rc;
    int flag = 0;
    H4B_CUDA_TRY(cudaMemcpyAsync(&flag, error, sizeof(int), cudaMemcpyDeviceToHost, s));
    H4B_CUDA_TRY(cudaStreamSynchronize(s));
    *host_error = flag;
    return flag ? H4B_EINVAL : 0;
}

extern "C" int h4b_rows_to_int4(const void* source, int source_dtype, int rows, int width, uint8_t* packed,
                                float* scales, void* stream) {
    using namespace h4b;
    if (!source || !packed || !scales || rows < 1 || width < 2 || (width & 1)) return H4B_EINVAL;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int grid = std::max(1, std::min((rows + 7) / 8, 8 * sm_count()));
    if (source_dtype == 0)
        rows_to_int4_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(source), rows, width, packed, scales);
    else if (source_dtype == 1)
        rows_to_int4_kernel<__half><<<grid, 256, 0, s>>>(static_cast<const __half*>(source), rows, width, packed,
                                                           scales);
    else
        return H4B_EINVAL;
    H4B_CUDA_TRY(cudaGetLastError());
    return 0;
}
