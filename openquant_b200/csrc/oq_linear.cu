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

// Per-(row, group) multipliers of dq_word: s * 16^-p for the nibble
// positions p the word is split into, and -8s.
struct DqScale {
    float2 mul[4];
    float2 m8s;
    bool fast;  // s * 2^-16 is a normal float and 8s is finite
};

__device__ __forceinline__ DqScale make_dq_scale(float s) {
    DqScale d;
    const float s4 = s * 0.0625f, s8 = s * 0.00390625f, s12 = s * 0.000244140625f, s16 = s * 1.52587890625e-05f;
    d.mul[0] = make_float2(s, s4);
    d.mul[1] = make_float2(s8, s12);
    d.mul[2] = make_float2(s16, s8);
    d.mul[3] = make_float2(s12, s16);
    d.m8s = make_float2(-8.0f * s, -8.0f * s);
    const float a = fabsf(s);
    d.fast = (a >= 0x1p-100f && a <= 0x1p100f);
    return d;
}

// Eight weights of one packed word (raw two's-complement nibbles, element i
// in bits 4i..4i+3) -> four packed pairs {w(2j), w(2j+1)} of
// round_x(fl32(q * s)).  The nibbles are lifted into fp32 as 2^23 + u*16^p
// (u = q + 8, offset binary, p = the nibble's position after at most one
// 12-bit shift) by AND/XOR into the 0x4B000000 exponent; subtracting 2^23 is
// exact, and fma(u*16^p, s*16^-p, -8s) is the exact value (u - 8) * s = q * s
// rounded once -- the reference's fp32 product.  Blackwell's packed
// f32x2 add/fma do two weights per instruction.  Scales whose 16^-4 multiple
// would be subnormal (or non-finite) take the per-nibble path.
template <typename XT>
__device__ __forceinline__ void dq_word(uint32_t w, const DqScale &sc, float s, uint32_t (&h)[4]) {
    if (sc.fast) {
        const uint32_t wh = w >> 12;
        const float f0 = __uint_as_float((w & 0x0000000Fu) ^ 0x4B000008u);
        const float f1 = __uint_as_float((w & 0x000000F0u) ^ 0x4B000080u);
        const float f2 = __uint_as_float((w & 0x00000F00u) ^ 0x4B000800u);
        const float f3 = __uint_as_float((w & 0x0000F000u) ^ 0x4B008000u);
        const float f4 = __uint_as_float((w & 0x000F0000u) ^ 0x4B080000u);
        const float f5 = __uint_as_float((wh & 0x00000F00u) ^ 0x4B000800u);
        const float f6 = __uint_as_float((wh & 0x0000F000u) ^ 0x4B008000u);
        const float f7 = __uint_as_float((wh & 0x000F0000u) ^ 0x4B080000u);
        const float2 m23 = make_float2(-8388608.0f, -8388608.0f);
        const float2 w01 = __ffma2_rn(__fadd2_rn(make_float2(f0, f1), m23), sc.mul[0], sc.m8s);
        const float2 w23 = __ffma2_rn(__fadd2_rn(make_float2(f2, f3), m23), sc.mul[1], sc.m8s);
        const float2 w45 = __ffma2_rn(__fadd2_rn(make_float2(f4, f5), m23), sc.mul[2], sc.m8s);
        const float2 w67 = __ffma2_rn(__fadd2_rn(make_float2(f6, f7), m23), sc.mul[3], sc.m8s);
        h[0] = XTraits<XT>::pack(w01.x, w01.y);
        h[1] = XTraits<XT>::pack(w23.x, w23.y);
        h[2] = XTraits<XT>::pack(w45.x, w45.y);
        h[3] = XTraits<XT>::pack(w67.x, w67.y);
    } else {
        const uint32_t u = w ^ 0x88888888u;
#pragma unroll
        for (int j = 0; j < 4; ++j) h[j] = XTraits<XT>::pack(dq(u, 2 * j, s), dq(u, 2 * j + 1, s));
    }
}

// ------------------------------------------------------------- GEMV ----
//
// One CTA = 16 weight rows x the whole K, split over WARPS warps: 128-column
// chunks are dealt round-robin to the warps and their partial sums reduced
// through shared memory in a fixed order (deterministic results).
//
// Memory-level parallelism: each warp keeps U chunks of packed weights in
// flight in a register ring (a chunk = 2 rows x 16 bytes per lane), and the
// first U loads are issued before griddepcontrol.wait, so under programmatic
// dependent launch they overlap the previous kernel's tail (weights never
// depend on it; x and y are touched only after the wait).
//
// Tensor cores: lane (g, t) (g = lane/4, t = lane%4) owns rows g and g+8 and
// columns 128*chunk + 32*t .. +32 and feeds mma.m16n8k16 with the weight tile
// as A (16 rows x 16 "slots") and x^T as B (slots x 8 batch columns).  The
// k-slots {2t, 2t+1, 2t+8, 2t+9} of a lane carry four consecutive real
// columns of its own segment, and B is loaded with the same permutation, so
// the tensor-core sum over slots is the sum over real columns.  NT n-tiles
// cover M <= 8*NT.  x is staged in shared memory when it fits (XS).
template <typename XT, int NT, int WARPS, int U, bool XS>
__global__ void __launch_bounds__(WARPS * 32) gemv_int4_kernel(const XT *__restrict__ x,
                                                               const uint8_t *__restrict__ packed,
                                                               const float *__restrict__ scales,
                                                               float *__restrict__ y, int m, int64_t n, int64_t k,
                                                               int64_t kp, int g) {
    extern __shared__ uint4 xs_raw[];
    __shared__ float red[WARPS][NT][4][32];
    const XT *xs = reinterpret_cast<const XT *>(xs_raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gi = lane >> 2, t = lane & 3;
    const int64_t row0 = (int64_t)blockIdx.x * 16;
    const int64_t ra = row0 + gi, rb = row0 + gi + 8;
    const bool va = ra < n, vb = rb < n;
    const int64_t groups = kp / g;
    const int64_t nchunks = cdiv(kp, 128);
    const uint8_t *pa = packed + ra * (kp / 2);
    const uint8_t *pb = packed + rb * (kp / 2);
    const float *sra = scales + ra * groups;
    const float *srb = scales + rb * groups;

    uint4 wa[U], wb[U];
    float sa[U], sb[U];
    auto load = [&](int u, int64_t c) {
        const int64_t k0 = 128 * c + 32 * t;
        wa[u] = make_uint4(0, 0, 0, 0);
        wb[u] = make_uint4(0, 0, 0, 0);
        sa[u] = 0.0f;
        sb[u] = 0.0f;
        if (c < nchunks && k0 < kp) {
            if (va) {
                wa[u] = __ldg(reinterpret_cast<const uint4 *>(pa + k0 / 2));
                sa[u] = __ldg(sra + k0 / g);
            }
            if (vb) {
                wb[u] = __ldg(reinterpret_cast<const uint4 *>(pb + k0 / 2));
                sb[u] = __ldg(srb + k0 / g);
            }
        }
    };
#pragma unroll
    for (int u = 0; u < U; ++u) load(u, warp + (int64_t)u * WARPS);

    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");

    if (XS) {  // stage x [m][k] (k % 8 == 0) in shared memory
        const int64_t vecs = (int64_t)m * k / 8;
        for (int64_t i = threadIdx.x; i < vecs; i += blockDim.x)
            xs_raw[i] = __ldg(reinterpret_cast<const uint4 *>(x) + i);
        __syncthreads();
    }

    float acc[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;

    const int64_t mine = nchunks > warp ? cdiv(nchunks - warp, WARPS) : 0;  // chunks of this warp
    for (int64_t base = 0; base < mine; base += U) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t c = warp + (base + u) * WARPS;
            if (base + u < mine) {
                const int k0 = (int)(128 * c + 32 * t);
                const uint32_t qa[4] = {wa[u].x, wa[u].y, wa[u].z, wa[u].w};
                const uint32_t qb[4] = {wb[u].x, wb[u].y, wb[u].z, wb[u].w};
                const DqScale dsa = make_dq_scale(sa[u]), dsb = make_dq_scale(sb[u]);
#pragma unroll
                for (int wd = 0; wd < 4; ++wd) {
                    const int kw = k0 + 8 * wd;  // columns kw..kw+7
                    uint4 xb[NT];
#pragma unroll
                    for (int j = 0; j < NT; ++j) {
                        const int mb = 8 * j + gi;
                        if (mb < m && kw < k)
                            xb[j] = XS ? *reinterpret_cast<const uint4 *>(xs + mb * (int)k + kw)
                                       : __ldg(reinterpret_cast<const uint4 *>(x + (int64_t)mb * k + kw));
                        else
                            xb[j] = make_uint4(0, 0, 0, 0);
                    }
                    uint32_t ha[4], hb[4];
                    dq_word<XT>(qa[wd], dsa, sa[u], ha);
                    dq_word<XT>(qb[wd], dsb, sb[u], hb);
                    // k16 step 0: nibbles 0-3 (pairs 0, 1); step 1: nibbles 4-7.
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
#pragma unroll
                        for (int j = 0; j < NT; ++j) {
                            const uint32_t b0 = h == 0 ? xb[j].x : xb[j].z;
                            const uint32_t b1 = h == 0 ? xb[j].y : xb[j].w;
                            XTraits<XT>::mma(acc[j], ha[2 * h], hb[2 * h], ha[2 * h + 1], hb[2 * h + 1], b0, b1);
                        }
                    }
                }
            }
            load(u, warp + (base + u + U) * WARPS);  // refill the slot
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

// Launch with programmatic stream serialization: a GEMV that follows
// another kernel in the stream may start (and prefetch its weights) while
// that kernel drains.  Without a preceding PDL-aware kernel it behaves like a
// normal launch.
template <typename Kern, typename XT>
int launch_pdl(Kern kern, unsigned blocks, unsigned threads, size_t smem, cudaStream_t st, const XT *x,
               const uint8_t *packed, const float *scales, float *y, int m, int64_t n, int64_t k, int64_t kp, int g) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t err = cudaLaunchKernelEx(&cfg, kern, x, packed, scales, y, m, n, k, kp, g);
    if (err != cudaSuccess) {
        set_error("int4_linear (GEMV): launch failed: %s", cudaGetErrorString(err));
        return OQ_ERR_CUDA;
    }
    return OQ_OK;
}

template <typename XT, int NT, int WARPS, int U>
int launch_gemv_t(const XT *x, const uint8_t *packed, const float *scales, float *y, int64_t m, int64_t n,
                  int64_t k, int64_t kp, int g, cudaStream_t st) {
    const unsigned blocks = (unsigned)cdiv(n, 16);
    const size_t xbytes = (size_t)m * (size_t)k * sizeof(XT);
    if (xbytes <= 48 * 1024 - sizeof(float) * WARPS * NT * 128)
        return launch_pdl(gemv_int4_kernel<XT, NT, WARPS, U, true>, blocks, WARPS * 32, xbytes, st, x, packed,
                          scales, y, (int)m, n, k, kp, g);
    return launch_pdl(gemv_int4_kernel<XT, NT, WARPS, U, false>, blocks, WARPS * 32, 0, st, x, packed, scales, y,
                      (int)m, n, k, kp, g);
}

template <typename XT>
int launch_gemv(const XT *x, const uint8_t *packed, const float *scales, float *y, int64_t m, int64_t n, int64_t k,
                int64_t kp, int g, cudaStream_t st) {
    switch ((m + 7) / 8) {
        case 1: return launch_gemv_t<XT, 1, 8, 4>(x, packed, scales, y, m, n, k, kp, g, st);
        case 2: return launch_gemv_t<XT, 2, 8, 4>(x, packed, scales, y, m, n, k, kp, g, st);
        case 3: case 4: return launch_gemv_t<XT, 4, 8, 2>(x, packed, scales, y, m, n, k, kp, g, st);
        default: return launch_gemv_t<XT, 8, 8, 2>(x, packed, scales, y, m, n, k, kp, g, st);
    }
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
