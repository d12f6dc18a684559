// Fused groupwise-INT4 dequant + matmul for the decode side (M <= 64) and a
// CUDA-core kernel for every other shape; oq_int4_linear() dispatches.
//
// Numerics (all kernels): the weight is w = round_x(fl32(q * s)) -- the fp32
// product of the signed nibble and its group scale, rounded to the
// activation type, as openquant/triton_int4.py:62-65 does -- and x * w is
// accumulated in fp32.  fl32(q*s) is formed exactly: q = (2^23 + u) -
// (2^23 + 8) with u the offset-binary nibble is exact, then one fp32 multiply.
#include "oq_common.cuh"

namespace oq {

int gemm_tcgen05_supported(int64_t m, int64_t n, int64_t k, int g, const void *x, const uint8_t *packed,
                           const float *y);
int gemm_tcgen05_launch(const void *x, int x_dtype, const uint8_t *packed, const float *scales, float *y,
                        int64_t m, int64_t n, int64_t k, int g, cudaStream_t st);

namespace {

template <typename XT> struct XTraits;
template <> struct XTraits<__half> {
    static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
        __half2 h = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<uint32_t *>(&h);
    }
    static __device__ __forceinline__ float round(float v) { return __half2float(__float2half_rn(v)); }
    static __device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
    static __device__ __forceinline__ void mma(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};\n"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    }
};
template <> struct XTraits<__nv_bfloat16> {
    static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
        __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<uint32_t *>(&h);
    }
    static __device__ __forceinline__ float round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
    static __device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
    static __device__ __forceinline__ void mma(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};\n"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    }
};

// fl32(q * s) for nibble i of `word`, where `word` has already been XORed
// with 0x88888888 (two's complement -> offset binary u = q + 8).
__device__ __forceinline__ float dq(uint32_t word, int i, float s) {
    const float f = __uint_as_float(0x4B000000u | ((word >> (4 * i)) & 15u));  // 2^23 + u
    return __fmul_rn(__fsub_rn(f, 8388616.0f), s);                               // (u - 8) * s
}

// ------------------------------------------------------------- GEMV ----
//
// One CTA = 16 weight rows x the whole K, split over WARPS warps (chunks of
// 128 columns dealt round-robin, partial sums reduced through shared memory
// in a fixed order, so results are deterministic).  In a warp, lane (g, t)
// (g = lane/4, t = lane%4) loads 16 bytes = 32 columns of rows g and g+8 at
// column 128*chunk + 32*t and feeds them to mma.m16n8k16 with the weight tile
// as the A operand (16 rows x 16 "slots") and x^T as B (slots x 8 batch
// columns).  The k-slots {2t, 2t+1, 2t+8, 2t+9} of a lane carry four
// consecutive real columns of its own 32-column segment; the B fragment is
// loaded with the same permutation, so the tensor-core sum over slots is the
// sum over real columns.  NT n-tiles cover M <= 8*NT.
template <typename XT, int NT, int WARPS>
__global__ void __launch_bounds__(WARPS * 32) gemv_int4_kernel(const XT *__restrict__ x,
                                                               const uint8_t *__restrict__ packed,
                                                               const float *__restrict__ scales,
                                                               float *__restrict__ y, int m, int64_t n, int64_t k,
                                                               int64_t kp, int g) {
    __shared__ float red[WARPS][NT][4][32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gi = lane >> 2, t = lane & 3;
    const int64_t row0 = (int64_t)blockIdx.x * 16;
    const int64_t ra = row0 + gi, rb = row0 + gi + 8;
    const bool va = ra < n, vb = rb < n;
    const int64_t groups = kp / g;
    const int64_t nchunks = cdiv(kp, 128);
    const uint8_t *pa = packed + ra * (kp / 2);
    const uint8_t *pb = packed + rb * (kp / 2);

    float acc[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;

    for (int64_t c = warp; c < nchunks; c += WARPS) {
        const int64_t k0 = 128 * c + 32 * t;  // first column of this lane's segment
        uint4 wa = make_uint4(0, 0, 0, 0), wb = make_uint4(0, 0, 0, 0);
        float sa = 0.0f, sb = 0.0f;
        if (k0 < kp) {
            if (va) {
                wa = __ldg(reinterpret_cast<const uint4 *>(pa + k0 / 2));
                sa = __ldg(scales + ra * groups + k0 / g);
            }
            if (vb) {
                wb = __ldg(reinterpret_cast<const uint4 *>(pb + k0 / 2));
                sb = __ldg(scales + rb * groups + k0 / g);
            }
        }
        const uint32_t wa4[4] = {wa.x ^ 0x88888888u, wa.y ^ 0x88888888u, wa.z ^ 0x88888888u, wa.w ^ 0x88888888u};
        const uint32_t wb4[4] = {wb.x ^ 0x88888888u, wb.y ^ 0x88888888u, wb.z ^ 0x88888888u, wb.w ^ 0x88888888u};
#pragma unroll
        for (int wd = 0; wd < 4; ++wd) {
            const int64_t kw = k0 + 8 * wd;  // columns kw..kw+7
            // B fragments: x[batch][kw..kw+7] for batch = 8*j + gi.
            uint4 xb[NT];
#pragma unroll
            for (int j = 0; j < NT; ++j) {
                const int mb = 8 * j + gi;
                xb[j] = (mb < m && kw < k) ? __ldg(reinterpret_cast<const uint4 *>(x + (int64_t)mb * k + kw))
                                           : make_uint4(0, 0, 0, 0);
            }
            // Two k16 steps per word: nibbles 0-3, then 4-7.
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint32_t a0 = XTraits<XT>::pack(dq(wa4[wd], 4 * h, sa), dq(wa4[wd], 4 * h + 1, sa));
                const uint32_t a2 = XTraits<XT>::pack(dq(wa4[wd], 4 * h + 2, sa), dq(wa4[wd], 4 * h + 3, sa));
                const uint32_t a1 = XTraits<XT>::pack(dq(wb4[wd], 4 * h, sb), dq(wb4[wd], 4 * h + 1, sb));
                const uint32_t a3 = XTraits<XT>::pack(dq(wb4[wd], 4 * h + 2, sb), dq(wb4[wd], 4 * h + 3, sb));
#pragma unroll
                for (int j = 0; j < NT; ++j) {
                    const uint32_t b0 = h == 0 ? xb[j].x : xb[j].z;
                    const uint32_t b1 = h == 0 ? xb[j].y : xb[j].w;
                    XTraits<XT>::mma(acc[j], a0, a1, a2, a3, b0, b1);
                }
            }
        }
    }

#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) red[warp][j][e][lane] = acc[j][e];
    __syncthreads();
    // Fixed-order reduction over warps; thread (j, e, lane) owns one output.
    for (int idx = threadIdx.x; idx < NT * 4 * 32; idx += blockDim.x) {
        const int j = idx / 128, e = (idx / 32) % 4, ln = idx % 32;
        float v = 0.0f;
#pragma unroll
        for (int wv = 0; wv < WARPS; ++wv) v += red[wv][j][e][ln];
        const int g2 = ln >> 2, t2 = ln & 3;
        const int64_t row = row0 + g2 + (e >= 2 ? 8 : 0);
        const int mb = 8 * j + 2 * t2 + (e & 1);
        if (row < n && mb < m) y[(int64_t)mb * n + row] = v;
    }
}

// ------------------------------------------------------------- SIMT ----
//
// Any shape and any even group size: one warp per weight row, lanes stride
// over K, up to 8 batch rows per pass (more passes for larger M).
template <typename XT>
__global__ void __launch_bounds__(256) simt_int4_kernel(const XT *__restrict__ x, const uint8_t *__restrict__ packed,
                                                        const float *__restrict__ scales, float *__restrict__ y,
                                                        int64_t m, int64_t n, int64_t k, int64_t kp, int g) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int64_t groups = kp / g;
    for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < n; row += warps) {
        const uint8_t *prow = packed + row * (kp / 2);
        for (int64_t m0 = 0; m0 < m; m0 += 8) {
            float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            for (int64_t c = lane; c < k; c += 32) {
                const int q = nibble_value(prow[c >> 1], (int)(c & 1));
                const float w = XTraits<XT>::round(__fmul_rn((float)q, scales[row * groups + c / g]));
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    if (m0 + i < m) acc[i] = fmaf(XTraits<XT>::to_f32(x[(m0 + i) * k + c]), w, acc[i]);
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                float v = acc[i];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                if (lane == 0 && m0 + i < m) y[(m0 + i) * n + row] = v;
            }
        }
    }
}

template <typename XT>
int launch_gemv(const XT *x, const uint8_t *packed, const float *scales, float *y, int64_t m, int64_t n, int64_t k,
                int64_t kp, int g, cudaStream_t st) {
    constexpr int W = 8;
    const unsigned blocks = (unsigned)cdiv(n, 16);
    switch ((m + 7) / 8) {
        case 1: gemv_int4_kernel<XT, 1, W><<<blocks, W * 32, 0, st>>>(x, packed, scales, y, (int)m, n, k, kp, g); break;
        case 2: gemv_int4_kernel<XT, 2, W><<<blocks, W * 32, 0, st>>>(x, packed, scales, y, (int)m, n, k, kp, g); break;
        case 3: case 4: gemv_int4_kernel<XT, 4, W><<<blocks, W * 32, 0, st>>>(x, packed, scales, y, (int)m, n, k, kp, g); break;
        default: gemv_int4_kernel<XT, 8, W><<<blocks, W * 32, 0, st>>>(x, packed, scales, y, (int)m, n, k, kp, g); break;
    }
    return check_launch("int4_linear (GEMV)");
}

template <typename XT>
int launch_simt(const XT *x, const uint8_t *packed, const float *scales, float *y, int64_t m, int64_t n, int64_t k,
                int64_t kp, int g, cudaStream_t st) {
    int64_t blocks = cdiv(n, 8);
    const int64_t cap = (int64_t)sm_count() * 8;
    if (blocks > cap) blocks = cap;
    simt_int4_kernel<XT><<<(unsigned)blocks, 256, 0, st>>>(x, packed, scales, y, m, n, k, kp, g);
    return check_launch("int4_linear (SIMT)");
}

}  // namespace

bool gemv_supported(int64_t m, int64_t k, int g, const void *x, const uint8_t *packed) {
    return m >= 1 && m <= 64 && g % 32 == 0 && k % 8 == 0 && aligned(x, 16) && aligned(packed, 16);
}

}  // namespace oq

using namespace oq;

extern "C" int oq_int4_linear(const void *x, int x_dtype, const uint8_t *packed, const float *scales, float *y,
                              int64_t m, int64_t n, int64_t k, int group_size, int kernel, int split_k,
                              oq_stream_t stream) {
    (void)split_k;
    clear_error();
    OQ_REQUIRE(x_dtype == OQ_F16 || x_dtype == OQ_BF16, "Input must be a 2D FP16 or BF16 tensor");
    OQ_REQUIRE(group_size >= 2 && group_size % 2 == 0, "Group size must be even and >= 2");
    OQ_REQUIRE(m >= 1 && n >= 1 && k >= 1, "Matrix dimensions must be positive");
    OQ_REQUIRE(x && packed && scales && y, "null pointer argument");
    const int64_t kp = cdiv(k, group_size) * group_size;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const bool gemv_ok = gemv_supported(m, k, group_size, x, packed);
    int which = kernel;
    if (which == OQ_KERNEL_AUTO) {
        if (gemv_ok && m <= 64)
            which = OQ_KERNEL_GEMV;
        else if (gemm_tcgen05_supported(m, n, k, group_size, x, packed, y))
            which = OQ_KERNEL_TCGEN05;
        else
            which = OQ_KERNEL_SIMT;
    }
    switch (which) {
        case OQ_KERNEL_GEMV:
            OQ_REQUIRE(gemv_ok, "GEMV kernel needs M <= 64, group_size % 32 == 0, K % 8 == 0 and 16-byte aligned x/packed");
            if (x_dtype == OQ_F16)
                return launch_gemv(static_cast<const __half *>(x), packed, scales, y, m, n, k, kp, group_size, st);
            return launch_gemv(static_cast<const __nv_bfloat16 *>(x), packed, scales, y, m, n, k, kp, group_size, st);
        case OQ_KERNEL_TCGEN05:
            OQ_REQUIRE(gemm_tcgen05_supported(m, n, k, group_size, x, packed, y),
                       "tcgen05 kernel does not support this shape/alignment");
            return gemm_tcgen05_launch(x, x_dtype, packed, scales, y, m, n, k, group_size, st);
        case OQ_KERNEL_SIMT:
            if (x_dtype == OQ_F16)
                return launch_simt(static_cast<const __half *>(x), packed, scales, y, m, n, k, kp, group_size, st);
            return launch_simt(static_cast<const __nv_bfloat16 *>(x), packed, scales, y, m, n, k, kp, group_size, st);
        default:
            return invalid("unknown kernel selector %d", kernel);
    }
}
