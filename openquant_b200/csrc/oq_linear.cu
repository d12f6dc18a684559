// Fused groupwise-INT4 dequant + matmul for the decode side (M <= 64) and a
// CUDA-core kernel for every other shape; oq_int4_linear() dispatches.
//
// Numerics (all kernels): the weight is w = round_x(fl32(q * s)) -- the fp32
// product of the signed nibble and its group scale, rounded to the
// activation type, as openquant/triton_int4.py:62-65 does -- and x * w is
// accumulated in fp32.  fl32(q*s) is formed exactly: q = (2^23 + u) -
// (2^23 + 8) with u the offset-binary nibble is exact, then one fp32 multiply.
#include "oq_dequant.cuh"
#include "oq_sm100.cuh"

#include <mutex>
#include <set>

namespace oq {

int gemm_tcgen05_supported(int64_t m, int64_t n, int64_t k, int g, const void *x, const uint8_t *packed,
                           const float *y);
int gemm_tcgen05_launch(const void *x, int x_dtype, const uint8_t *packed, const float *scales, OutSpec y,
                        int64_t m, int64_t n, int64_t k, int g, void *ws, size_t ws_bytes, cudaStream_t st,
                        int64_t gate_n = 0);
size_t gemm_tcgen05_workspace_bytes(int64_t m, int64_t n, int64_t k, int g);

namespace {

// One 128-column chunk of the GEMV: for each of the lane's four words, the
// B fragment (x) and the two k16 steps of dequant + mma.
template <typename XT, int NT, bool XS, bool FAST>
__device__ __forceinline__ void gemv_chunk(int c, const uint32_t (&qa)[4], const uint32_t (&qb)[4],
                                           const DqScale &dsa, const DqScale &dsb, const uint32_t (&xaddr)[NT],
                                           const bool (&xon)[NT], const XT *const (&xg)[NT], uint4 (&xb)[NT],
                                           float (&acc)[2][NT][4], int xo = 8) {
    // xo: x offset per word step -- 8 for lanes holding 32 consecutive
    // columns, 32 for the ldsm_x4 layout (see gemv_chunk_sa's TX)
#pragma unroll
    for (int wd = 0; wd < 4; ++wd) {
#pragma unroll
        for (int j = 0; j < NT; ++j) {
            if (XS) {
                const uint32_t addr = xaddr[j] + (uint32_t)(128 * c + xo * wd) * 2u;
                asm volatile(
                    "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                    " @p ld.shared.v4.u32 {%0, %1, %2, %3}, [%5];\n}\n"
                    : "+r"(xb[j].x), "+r"(xb[j].y), "+r"(xb[j].z), "+r"(xb[j].w)
                    : "r"((int)xon[j]), "r"(addr));
            } else if (xon[j]) {
                xb[j] = __ldg(reinterpret_cast<const uint4 *>(xg[j] + 128 * c + xo * wd));
            }
        }
        // k16 step 0: nibbles 0-3 (pairs 0, 1); step 1: nibbles 4-7.
        {
            uint32_t ha[2], hb[2];
            dq_half<XT, 0, FAST>(qa[wd], dsa, ha);
            dq_half<XT, 0, FAST>(qb[wd], dsb, hb);
#pragma unroll
            for (int j = 0; j < NT; ++j)
                XTraits<XT>::mma(acc[0][j], ha[0], hb[0], ha[1], hb[1], xb[j].x, xb[j].y);
        }
        {
            uint32_t ha[2], hb[2];
            dq_half<XT, 1, FAST>(qa[wd], dsa, ha);
            dq_half<XT, 1, FAST>(qb[wd], dsb, hb);
#pragma unroll
            for (int j = 0; j < NT; ++j)
                XTraits<XT>::mma(acc[1][j], ha[0], hb[0], ha[1], hb[1], xb[j].z, xb[j].w);
        }
    }
}

// Padding (fp16 elements) after each staged x row: rows then start 16 banks
// apart, so the 8 lanes of a quarter-warp (rows g, g + 1 x 4 column
// offsets 8 t) read distinct banks.
constexpr int kXPad = 32;
// The TMA-fed GEMVs use that layout when a chunk lies in one scale group (g
// >= 128); otherwise, and in the register-ring kernel, lanes read x at 32 t +
// 8 wd, where 8 elements of padding spread the rows best.
inline int gemv_xpad(int g) { return g >= 128 ? kXPad : 8; }

// Bytes of the GEMV's double-buffered cross-warp reduction buffer.
__host__ __device__ constexpr size_t gemv_red_bytes(int warps, int nt) { return 2u * warps * nt * 4 * 32 * 4; }

// Scale-after variant of gemv_chunk (fp16 x, whole 128-column chunk in one
// group): nibbles become exact fp16 integers and the group scale is applied
// to the chunk's fp32 partial sums.  Per packed word W the LOP3 magic
// (W & 0x000F000F) ^ 0x64086408 is the half pair (1024 + u0, 1024 + u4),
// u = n ^ 8 the offset-binary nibble; the 0x00F000F0 mask gives
// (1024 + 16 u1, 1024 + 16 u5), and W >> 8 the same for nibbles 2, 6 and 3,
// 7.  One HSUB2 of 1032 (or 1024 + 128) leaves q (or 16 q) exactly.  The
// "class 0" k16 step takes nibbles {0,4,2,6}, the "class 1" step nibbles
// {1,5,3,7} (16 q); x is staged in the matching order with the class-1
// halves divided by 16 (sa_perm_x), so one 16-byte load gives both steps' B
// fragments and both steps accumulate q * x into the same fp32 sums.
// Products of fp16 q and x are exact (x / 16 too, unless it falls below the
// fp16 normal range, |x| < 2^-10) and the tensor core sums them in fp32;
// y += s * sum per chunk.
// Scales (rows g and g + 8, col) of a stage's scale box.  When a stage row is exactly 128
// bytes (32 groups: g = 128) the box arrives 128-byte swizzled (16-byte
// unit u of row r stored at u ^ (r % 8), make_gemv_maps), so the 8 rows a
// warp reads at one column fall in 8 bank groups instead of one.
// Rows g and g + 8 share (row % 8), hence the swizzled column: both scales
// of a lane come from one index computation.
// One group scale from global memory: fp32 (the reference's format) or, with
// half_scales, fp16 (the fp16-scale variant; `scales` then points at halves).
__device__ __forceinline__ float load_scale(const float *scales, size_t idx, int half_scales) {
    return half_scales ? __half2float(__ldg(reinterpret_cast<const __half *>(scales) + idx)) : __ldg(scales + idx);
}

__device__ __forceinline__ void stage_scales(const float *sst, int gi, int col, int spr, float &sa, float &sb) {
    const int c = spr == 32 ? ((((col >> 2) ^ (gi & 7)) << 2) | (col & 3)) : col;
    sa = sst[gi * spr + c];
    sb = sst[(gi + 8) * spr + c];
}

// Four 8x8 b16 matrices from shared memory (ldmatrix): lane L gives the
// address of row L % 8 of matrix L / 8 and receives, from each matrix j,
// the 32-bit word L % 4 of row L / 4 in r[j].  On the 128-byte-swizzled
// weight stages the 8 rows of one logical 16-byte unit lie in 8 distinct
// bank groups, so the load is free of bank conflicts (a per-lane 16-byte
// load of rows g, g+1 x 4 units is not: both rows' units share banks).
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr)
                 : "memory");
}

__device__ __forceinline__ uint32_t lop3_and_xor(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
    __half2 r = __hsub2(*reinterpret_cast<__half2 *>(&a), *reinterpret_cast<__half2 *>(&b));
    return *reinterpret_cast<uint32_t *>(&r);
}

// Eight fp16 x values in natural order -> the scale-after layout:
// (x0, x4) (x2, x6) for the class-0 step, (x1, x5)/16 (x3, x7)/16 for the
// class-1 step (whose dequantized weights are 16 q).
__device__ __forceinline__ uint4 sa_perm_x(uint4 v) {
    uint32_t z = __byte_perm(v.x, v.z, 0x7632), w = __byte_perm(v.y, v.w, 0x7632);
    const __half2 k = __float2half2_rn(0.0625f);
    __half2 hz = __hmul2(*reinterpret_cast<__half2 *>(&z), k), hw = __hmul2(*reinterpret_cast<__half2 *>(&w), k);
    return make_uint4(__byte_perm(v.x, v.z, 0x5410), __byte_perm(v.y, v.w, 0x5410),
                      *reinterpret_cast<uint32_t *>(&hz), *reinterpret_cast<uint32_t *>(&hw));
}

// x [m][k] -> xs [m][xstride] (zero beyond k; SA: the scale-after layout).
// FOLD also fills corr[c][r] (r < m, 128-column chunk c) = 1032 * (sum of the
// chunk's class-0 x of row r) + 1152 * (sum of its class-1 x / 16), in a fixed
// order: with KP % 128 == 0, thread i stages vector i % (KP/8) of row
// i / (KP/8), so a chunk's 16 vectors lie in 16 aligned lanes and a
// shuffle tree sums them.  All threads of the block call it.
template <typename XT, bool SA, bool FOLD, int U = 1>
__device__ __forceinline__ void gemv_stage_x(const XT *__restrict__ x, XT *xs, float *corr, int m, int k, int kp,
                                             int xstride, int nthreads) {
    // U vectors per thread per pass, their loads issued first: a pass waits
    // for one round trip to L2 instead of U (the persistent TMA kernel stages
    // 8-32 vectors per thread at M = 4-16, K = 4096; the register-capped tile
    // and pair kernels use U = 1).
    if (!FOLD) {
        const int rowv = xstride / 8, kv = k / 8, total = m * rowv;
        for (int i0 = threadIdx.x; i0 < total; i0 += U * nthreads) {
            uint4 v[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int i = i0 + u * nthreads;
                const int r = i / rowv, c = i - r * rowv;
                v[u] = i < total && c < kv ? __ldg(reinterpret_cast<const uint4 *>(x) + (size_t)r * kv + c)
                                           : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int i = i0 + u * nthreads;
                if (i < total) reinterpret_cast<uint4 *>(xs)[i] = SA ? sa_perm_x(v[u]) : v[u];
            }
        }
    } else {
        const int kv8 = kp / 8, kv = k / 8, total = m * kv8;
        for (int b0 = (int)threadIdx.x - (int)(threadIdx.x & 31); b0 < total; b0 += U * nthreads) {
            uint4 v[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int i = b0 + u * nthreads + (int)(threadIdx.x & 31);
                const int r = i < total ? i / kv8 : 0, cv = i < total ? i - r * kv8 : 0;
                v[u] = make_uint4(0, 0, 0, 0);
                if (i < total && cv < kv) v[u] = __ldg(reinterpret_cast<const uint4 *>(x) + (size_t)r * kv + cv);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int i = b0 + u * nthreads + (int)(threadIdx.x & 31);
                const bool live = i < total;
                const int r = live ? i / kv8 : 0, cv = live ? i - r * kv8 : 0;
                const uint4 w = sa_perm_x(v[u]);
                if (live) reinterpret_cast<uint4 *>(xs)[r * (xstride / 8) + cv] = w;
                const float2 f0 = __half22float2(*reinterpret_cast<const __half2 *>(&w.x));
                const float2 f1 = __half22float2(*reinterpret_cast<const __half2 *>(&w.y));
                const float2 f2 = __half22float2(*reinterpret_cast<const __half2 *>(&w.z));
                const float2 f3 = __half22float2(*reinterpret_cast<const __half2 *>(&w.w));
                float t = 1032.0f * ((f0.x + f0.y) + (f1.x + f1.y)) + 1152.0f * ((f2.x + f2.y) + (f3.x + f3.y));
#pragma unroll
                for (int o = 8; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
                if (live && (cv & 15) == 0) corr[(cv >> 4) * 16 + r] = t;
            }
        }
    }
}

// The part of x one warp of the pair GEMV reads -- its chunks c = wg + 8 q
// (q < 4, c < nchunks) of every row r < m -- staged as gemv_stage_x does
// (same layout, same bias table entries, same summation order), so the warp
// can start on its chunks after a __syncwarp instead of a barrier over the
// whole CTA: the other warps' x loads no longer gate it.  Lane l stages
// vectors l and l + 32 of the warp's 64 per row (chunk q = vector / 16), RP
// rows per pass with all their loads issued first (one L2 round trip per RP
// rows).  Warps of the two tile groups with the same wg write the same
// values.
template <typename XT, bool SA, bool FOLD, int RP>
__device__ __forceinline__ void gemv_stage_x_warp(const XT *__restrict__ x, XT *xs, float *corr, int m, int k,
                                                  int xstride, int wg, int lane, int nchunks) {
    const int kv = k / 8;
    for (int r0 = 0; r0 < m; r0 += RP) {
        uint4 v[RP][2];
#pragma unroll
        for (int rr = 0; rr < RP; ++rr)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int r = r0 + rr, i = lane + 32 * h, c = wg + 8 * (i >> 4), cv = 16 * c + (i & 15);
                v[rr][h] = r < m && c < nchunks && cv < kv
                               ? __ldg(reinterpret_cast<const uint4 *>(x) + (size_t)r * kv + cv)
                               : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
        for (int rr = 0; rr < RP; ++rr) {
            if (r0 + rr >= m) break;  // warp-uniform
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int r = r0 + rr, i = lane + 32 * h, c = wg + 8 * (i >> 4), cv = 16 * c + (i & 15);
                const bool live = c < nchunks;
                const uint4 w = SA ? sa_perm_x(v[rr][h]) : v[rr][h];
                if (live) reinterpret_cast<uint4 *>(xs)[r * (xstride / 8) + cv] = w;
                if (FOLD) {  // warp-uniform: every lane takes part in the shuffles
                    const float2 f0 = __half22float2(*reinterpret_cast<const __half2 *>(&w.x));
                    const float2 f1 = __half22float2(*reinterpret_cast<const __half2 *>(&w.y));
                    const float2 f2 = __half22float2(*reinterpret_cast<const __half2 *>(&w.z));
                    const float2 f3 = __half22float2(*reinterpret_cast<const __half2 *>(&w.w));
                    float t = 1032.0f * ((f0.x + f0.y) + (f1.x + f1.y)) + 1152.0f * ((f2.x + f2.y) + (f3.x + f3.y));
#pragma unroll
                    for (int o = 8; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
                    if (live && (i & 15) == 0) corr[c * 16 + r] = t;
                }
            }
        }
    }
}

// FOLD (staged x only): the biased halves (1032 + q, 1152 + 16 q) go to the
// tensor core as they are -- no HSUB2 -- and the bias's share of each sum,
// 1032 * (sum of the chunk's class-0 x) + 1152 * (sum of its class-1 x / 16)
// for batch row n, is subtracted once per chunk: corr_ct points at
// corr[c][2t] of a [chunk][16 batch rows] table (gemv_fold_corr).  Products
// stay exact; the fp32 sums grow to ~1e3 |x|, so the result carries ~1e-3
// absolute error per chunk (~1e-5 relative in y), below the reference's own
// fp16 weight rounding.
// TX (weights loaded with ldsm_x4): a lane's word wd holds chunk columns
// 32 wd + 8 t .. + 7 instead of 32 t + 8 wd .. + 7, and x is read to match
// (xaddr / xg then point at column 8 t).
template <int NT, bool XS, bool FOLD = false, bool TX = false>
__device__ __forceinline__ void gemv_chunk_sa(int c, const uint32_t (&qa)[4], const uint32_t (&qb)[4], float sa,
                                              float sb, const uint32_t (&xaddr)[NT], const bool (&xon)[NT],
                                              const __half *const (&xg)[NT], uint4 (&xb)[NT],
                                              float (&acc)[2][NT][4], const float *corr_ct = nullptr) {
    static_assert(!FOLD || XS, "the bias correction needs staged x");
    float part[2][NT][4];  // one accumulator chain per nibble class
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int j = 0; j < NT; ++j) part[a][j][0] = part[a][j][1] = part[a][j][2] = part[a][j][3] = 0.0f;
    const uint32_t k1032 = 0x64086408u;  // half2 (1032, 1032)
    const uint32_t k1152 = 0x64806480u;  // half2 (1152, 1152)
#pragma unroll
    for (int wd = 0; wd < 4; ++wd) {
#pragma unroll
        for (int j = 0; j < NT; ++j) {
            if (XS) {
                const uint32_t addr = xaddr[j] + (uint32_t)(128 * c + (TX ? 32 : 8) * wd) * 2u;
                asm volatile(
                    "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                    " @p ld.shared.v4.u32 {%0, %1, %2, %3}, [%5];\n}\n"
                    : "+r"(xb[j].x), "+r"(xb[j].y), "+r"(xb[j].z), "+r"(xb[j].w)
                    : "r"((int)xon[j]), "r"(addr));
            } else if (xon[j]) {
                // natural order x0..x7 -> (x0,x4) (x2,x6) (x1,x5) (x3,x7)
                xb[j] = sa_perm_x(__ldg(reinterpret_cast<const uint4 *>(xg[j] + 128 * c + (TX ? 32 : 8) * wd)));
            }
        }
        const uint32_t wa = qa[wd], wb = qb[wd];
        const uint32_t wa8 = wa >> 8, wb8 = wb >> 8;
        // class 0: (q0, q4) and (q2, q6)
        {
            uint32_t a0 = lop3_and_xor(wa, 0x000F000Fu, 0x64086408u), a2 = lop3_and_xor(wa8, 0x000F000Fu, 0x64086408u);
            uint32_t b0 = lop3_and_xor(wb, 0x000F000Fu, 0x64086408u), b2 = lop3_and_xor(wb8, 0x000F000Fu, 0x64086408u);
            if (!FOLD) {
                a0 = hsub2_u32(a0, k1032), a2 = hsub2_u32(a2, k1032);
                b0 = hsub2_u32(b0, k1032), b2 = hsub2_u32(b2, k1032);
            }
#pragma unroll
            for (int j = 0; j < NT; ++j)
                XTraits<__half>::mma(part[0][j], a0, b0, a2, b2, xb[j].x, xb[j].y);
        }
        // class 1: (16 q1, 16 q5) and (16 q3, 16 q7)
        {
            uint32_t a1 = lop3_and_xor(wa, 0x00F000F0u, 0x64806480u), a3 = lop3_and_xor(wa8, 0x00F000F0u, 0x64806480u);
            uint32_t b1 = lop3_and_xor(wb, 0x00F000F0u, 0x64806480u), b3 = lop3_and_xor(wb8, 0x00F000F0u, 0x64806480u);
            if (!FOLD) {
                a1 = hsub2_u32(a1, k1152), a3 = hsub2_u32(a3, k1152);
                b1 = hsub2_u32(b1, k1152), b3 = hsub2_u32(b3, k1152);
            }
#pragma unroll
            for (int j = 0; j < NT; ++j)
                XTraits<__half>::mma(part[1][j], a1, b1, a3, b3, xb[j].z, xb[j].w);
        }
    }
    // D fragment: elements 0, 1 belong to row g (scale sa), 2, 3 to row g+8;
    // elements 0, 2 to batch row 8j + 2t, 1, 3 to 8j + 2t + 1.
#pragma unroll
    for (int j = 0; j < NT; ++j) {
        float c0 = 0.0f, c1 = 0.0f;
        if (FOLD) {
            const float2 cv = *reinterpret_cast<const float2 *>(corr_ct + 8 * j);
            c0 = cv.x, c1 = cv.y;
        }
        acc[0][j][0] = fmaf(part[0][j][0] + part[1][j][0] - c0, sa, acc[0][j][0]);
        acc[0][j][1] = fmaf(part[0][j][1] + part[1][j][1] - c1, sa, acc[0][j][1]);
        acc[0][j][2] = fmaf(part[0][j][2] + part[1][j][2] - c0, sb, acc[0][j][2]);
        acc[0][j][3] = fmaf(part[0][j][3] + part[1][j][3] - c1, sb, acc[0][j][3]);
    }
}

template <typename XT, int NT, int WARPS, int U, bool XS, int MINB, bool SA>
__global__ void __launch_bounds__(WARPS * 32, MINB) gemv_int4_kernel(const XT *__restrict__ x,
                                                               const uint8_t *__restrict__ packed,
                                                               const float *__restrict__ scales,
                                                               OutSpec y, int m, int n, int k, int kp,
                                                               int gshift, int xstride, int prefetch) {
    static_assert(!SA || std::is_same<XT, __half>::value, "scale-after mode is for fp16 x");
    // Dynamic shared memory: the double-buffered cross-warp reduction, then
    // the staged x.
    extern __shared__ uint4 smem_dyn[];
    auto red = reinterpret_cast<float(*)[WARPS][NT][4][32]>(smem_dyn);
    uint4 *xs_raw = smem_dyn + gemv_red_bytes(WARPS, NT) / 16;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gi = lane >> 2, t = lane & 3;
    const int nchunks = (kp + 127) >> 7;
    const int groups = kp >> gshift;
    const int tiles = (n + 15) >> 4;
    // This CTA's tiles: blockIdx.x, blockIdx.x + gridDim.x, ...; each warp
    // walks positions p = (tile i, its j-th chunk c = warp + j * WARPS).
    const int my_tiles = blockIdx.x < tiles ? (tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int cpw = (nchunks + WARPS - 1) / WARPS;  // chunk slots per warp per tile
    const int npos = my_tiles * cpw;

    // Refill cursor: the next position to load, as (tile ordinal, slot)
    // with row pointers recomputed only when the tile changes.
    int r_ti = 0, r_jj = 0;
    const uint8_t *r_pa = nullptr, *r_pb = nullptr;
    const float *r_sa = nullptr, *r_sb = nullptr;
    auto set_rows = [&](int ti) {
        const int row0 = ((int)blockIdx.x + ti * (int)gridDim.x) * 16;
        const int ra = min(row0 + gi, n - 1), rb = min(row0 + gi + 8, n - 1);
        r_pa = packed + (size_t)ra * (kp / 2) + 16 * t;
        r_pb = packed + (size_t)rb * (kp / 2) + 16 * t;
        r_sa = scales + (size_t)ra * groups;
        r_sb = scales + (size_t)rb * groups;
    };
    uint4 wa[U], wb[U];
    float sa[U], sb[U];
    // Loads the cursor's chunk into slot u and advances the cursor (past the
    // last position it keeps re-reading the last chunk, which is harmless).
    auto load = [&](int u) {
        const int c = min(warp + r_jj * WARPS, nchunks - 1);
        const int k0 = 128 * c + 32 * t;
        const bool in = k0 < kp;
        const int off = in ? 64 * c : -16 * t;
        const int sidx = in ? (k0 >> gshift) : 0;
        wa[u] = __ldg(reinterpret_cast<const uint4 *>(r_pa + off));
        wb[u] = __ldg(reinterpret_cast<const uint4 *>(r_pb + off));
        const float a = __ldg(r_sa + sidx);
        const float b = __ldg(r_sb + sidx);
        sa[u] = in ? a : 0.0f;
        sb[u] = in ? b : 0.0f;
        if (++r_jj == cpw && r_ti + 1 < my_tiles) {
            r_jj = 0;
            set_rows(++r_ti);
        } else if (r_jj == cpw) {
            r_jj = cpw - 1;  // stay on the last position
        }
    };
    // Dependent launches may start now; they wait for this grid before
    // touching anything it writes.  Weights are read before this grid's own
    // wait only with `prefetch` (static weights: written before any kernel
    // still in flight on the stream).
    asm volatile("griddepcontrol.launch_dependents;");
    if (!prefetch) asm volatile("griddepcontrol.wait;" ::: "memory");
    if (npos > 0) {
        set_rows(0);
#pragma unroll
        for (int u = 0; u < U; ++u) load(u);
    }
    if (prefetch) asm volatile("griddepcontrol.wait;" ::: "memory");
    if (npos == 0) return;

    if (XS) {  // x [m][k] -> xs [m][xstride] halves, zero beyond k
        const int rowv = xstride / 8, kv = k / 8;
        for (int i = threadIdx.x; i < m * rowv; i += blockDim.x) {
            const int r = i / rowv, c = i - r * rowv;
            uint4 v = c < kv ? __ldg(reinterpret_cast<const uint4 *>(x) + (size_t)r * kv + c) : make_uint4(0, 0, 0, 0);
            if (SA) {  // x0..x7 -> (x0,x4) (x2,x6) (x1,x5) (x3,x7)
                v = sa_perm_x(v);
            }
            xs_raw[i] = v;
        }
        __syncthreads();
    }
    // Per n-tile: this lane's batch row and whether it exists.
    uint32_t xaddr[NT];
    bool xon[NT];
    const XT *xg[NT];
#pragma unroll
    for (int j = 0; j < NT; ++j) {
        const int mb = 8 * j + gi;
        xon[j] = mb < m;
        const int mr = xon[j] ? mb : 0;
        xaddr[j] = (uint32_t)__cvta_generic_to_shared(xs_raw) + (uint32_t)(mr * xstride + 32 * t) * 2u;
        xg[j] = x + (size_t)mr * k + 32 * t;
    }
    uint4 xb[NT];
#pragma unroll
    for (int j = 0; j < NT; ++j) xb[j] = make_uint4(0, 0, 0, 0);

    // Two accumulator sets (even / odd k16 step) halve the mma dependency chain.
    float acc[2][NT][4];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int j = 0; j < NT; ++j) acc[a][j][0] = acc[a][j][1] = acc[a][j][2] = acc[a][j][3] = 0.0f;

    // Compute cursor: tile ordinal ti, slot jj (chunk c = warp + jj * WARPS).
    int ti = 0, jj = 0;
    for (int base = 0; base < npos; base += U) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if (base + u < npos) {
                const int c = warp + jj * WARPS;
                if (c < nchunks) {
                    const uint32_t qa[4] = {wa[u].x, wa[u].y, wa[u].z, wa[u].w};
                    const uint32_t qb[4] = {wb[u].x, wb[u].y, wb[u].z, wb[u].w};
                    if constexpr (SA) {
                        gemv_chunk_sa<NT, XS>(c, qa, qb, sa[u], sb[u], xaddr, xon, xg, xb, acc);
                    } else {
                        // One warp-uniform branch per chunk keeps the rare
                        // per-nibble path out of the hot loop.
                        const DqScale dsa = make_dq_scale(sa[u]), dsb = make_dq_scale(sb[u]);
                        if (__all_sync(0xffffffffu, dsa.fast && dsb.fast))
                            gemv_chunk<XT, NT, XS, true>(c, qa, qb, dsa, dsb, xaddr, xon, xg, xb, acc);
                        else
                            gemv_chunk<XT, NT, XS, false>(c, qa, qb, dsa, dsb, xaddr, xon, xg, xb, acc);
                    }
                }
                load(u);  // refill the slot: the next tile's chunks stream in
                if (++jj == cpw) {
                    // End of this CTA's tile ti: fixed-order reduction over warps.
                    const int buf = ti & 1;
#pragma unroll
                    for (int j = 0; j < NT; ++j)
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            red[buf][warp][j][e][lane] = acc[0][j][e] + acc[1][j][e];
                            acc[0][j][e] = 0.0f;
                            acc[1][j][e] = 0.0f;
                        }
                    __syncthreads();
                    const int row0 = ((int)blockIdx.x + ti * (int)gridDim.x) * 16;
                    for (int idx = threadIdx.x; idx < NT * 4 * 32; idx += blockDim.x) {
                        const int j = idx / 128, e = (idx / 32) % 4, ln = idx % 32;
                        float v = 0.0f;
#pragma unroll
                        for (int wv = 0; wv < WARPS; ++wv) v += red[buf][wv][j][e][ln];
                        const int g2 = ln >> 2, t2 = ln & 3;
                        const int row = row0 + g2 + (e >= 2 ? 8 : 0);
                        const int mb = 8 * j + 2 * t2 + (e & 1);
                        if (row < n && mb < m) y.store(mb, row, v);
                    }
                    jj = 0;
                    ++ti;
                }
            }
        }
    }
}

// ----------------------------------------------------------- TMA GEMV ----
//
// Persistent decode GEMV fed by TMA.  One CTA per SM loops over 16-row
// tiles; a tile's K is cut into stages of 128*CPW*CW columns (32 KB of
// packed weights: fewer, larger stages stream faster than many small ones).
// Warp CW (the producer) keeps a ring of S stages in flight: for each stage
// it waits for the slot to be empty, then one lane issues the stage's TMA
// boxes (16 rows x 128 bytes each, 128-byte swizzled) and, when the scales'
// row pitch allows it (groups % 4 == 0), one TMA box of the stage's scales,
// all completing on full[slot].  Consumer warp w takes the stage's chunks
// w, w + CW, ... (128 columns each): it reads its two 16-byte pieces per
// chunk (rows g and g+8) from the swizzled boxes conflict-free, runs the
// same dequant + mma as the register-ring kernel, and arrives on
// empty[slot].  At the end of a tile the consumer warps reduce their partial
// sums in a fixed order (named barrier 1, producer excluded).
//
// PDL: every CTA lets dependent launches start at once.  The consumers read
// x and write y after griddepcontrol.wait; the producer streams the weights
// and scales after it too, unless the caller declared them static
// (`prefetch`: written before any kernel still in flight on the stream), in
// which case they stream while the previous grid drains.
template <int CW, int CPW>
struct TmaGemvLayout {
    static constexpr int kStageCols = 128 * CW * CPW;  // columns per stage
    static constexpr int kStageBytes = 16 * kStageCols / 2;
    static constexpr int kBoxes = kStageBytes / 2048;  // 16 rows x 128 B boxes
};

template <typename XT, int NT, int CW, int CPW, bool SA, bool XS, bool STMA>
__global__ void __launch_bounds__((CW + 1) * 32, CW <= 8 ? 2 : 1)
    gemv_tma_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap smap,
                    const XT *__restrict__ x, const float *__restrict__ scales, OutSpec y, int m, int n,
                    int k, int kp, int gshift, int xstride, int nstages, int prefetch, int gate_n, int nred,
                    int half_scales) {
    static_assert(!SA || std::is_same<XT, __half>::value, "scale-after mode is for fp16 x");
    using L = TmaGemvLayout<CW, CPW>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte alignment for the swizzled boxes.
    uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    const int spr = L::kStageCols >> gshift;  // scales per row per stage
    const int sbytes = ((16 * spr * 4 + 127) / 128) * 128;
    uint8_t *wbuf = smem;                                               // [S][boxes][16][128]
    float *sbuf = reinterpret_cast<float *>(wbuf + (size_t)nstages * L::kStageBytes);  // [S][16][spr]
    uint64_t *full = reinterpret_cast<uint64_t *>(reinterpret_cast<uint8_t *>(sbuf) + (size_t)nstages * sbytes);
    uint64_t *empty = full + nstages;
    auto red = reinterpret_cast<float(*)[CW][NT][4][32]>(empty + nstages);  // [nred]
    XT *xs = reinterpret_cast<XT *>(reinterpret_cast<uint8_t *>(red) + gemv_red_bytes(CW, NT) / 2 * nred);
    constexpr bool FOLD = SA && XS;  // bias-folded dequantization (gemv_chunk_sa)
    float *corr = reinterpret_cast<float *>(xs + (size_t)m * xstride);  // [chunks][16]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int groups = kp >> gshift;
    // gate_n > 0 (SiLU-gate mode): the weights are the [gate; up] stack of
    // 2 gate_n rows; the CTA walks tile pairs u = blockIdx.x + j * gridDim.x,
    // gate tile u (rows 16u..) then up tile u (rows gate_n + 16u..), and
    // writes silu(gate) * up for the gate_n output features.
    static_assert(NT * 4 * 32 <= CW * 32, "one reduced output per thread and tile");
    const int units = gate_n ? (gate_n + 15) >> 4 : (n + 15) >> 4;
    const int my_units = (int)blockIdx.x < units ? (units - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int my_tiles = gate_n ? 2 * my_units : my_units;
    auto tile_row0 = [&](int ti) {
        return gate_n ? ((ti & 1) ? gate_n : 0) + ((int)blockIdx.x + (ti >> 1) * (int)gridDim.x) * 16
                      : ((int)blockIdx.x + ti * (int)gridDim.x) * 16;
    };
    const int nchunks = (kp + 127) >> 7;
    const int spt = (kp + L::kStageCols - 1) / L::kStageCols;  // stages per tile
    const int npos = my_tiles * spt;

    // Dependent launches may start now; they wait for this grid before
    // touching anything it writes (as in the ring kernel).
    asm volatile("griddepcontrol.launch_dependents;");
    if (threadIdx.x == 0) {
        for (int i = 0; i < nstages; ++i) {
            mbar_init(&full[i], 1);   // the producer's expect_tx arrival
            mbar_init(&empty[i], CW);  // one arrival per consumer warp
        }
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == CW) {  // ------------------------------------ producer
        if (lane == 0) {
            tma_prefetch_desc(&wmap);
            if (STMA) tma_prefetch_desc(&smap);
            if (!prefetch) asm volatile("griddepcontrol.wait;" ::: "memory");
            for (int pos = 0; pos < npos; ++pos) {
                const int slot = pos % nstages, round = pos / nstages;
                if (round > 0 && !mbar_wait(&empty[slot], (round - 1) & 1)) break;
                const int ti = pos / spt, st = pos - ti * spt;
                const int row0 = tile_row0(ti);
                const int k0 = st * L::kStageCols;
                mbar_arrive_expect_tx(&full[slot], L::kStageBytes + (STMA ? 16 * spr * (half_scales ? 2 : 4) : 0));
#pragma unroll
                for (int b = 0; b < L::kBoxes; ++b)
                    tma_load_2d(wbuf + (size_t)slot * L::kStageBytes + b * 2048, &wmap, &full[slot], k0 / 2 + 128 * b,
                                row0);
                if (STMA)
                    tma_load_2d(reinterpret_cast<uint8_t *>(sbuf) + (size_t)slot * sbytes, &smap, &full[slot],
                                k0 >> gshift, row0);
            }
        }
        return;
    }

    // ------------------------------------------------------ consumers
    const int gi = lane >> 2, t = lane & 3;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (XS) {
        gemv_stage_x<XT, SA, FOLD, 4>(x, xs, corr, m, k, kp, xstride, CW * 32);
        asm volatile("bar.sync 1, %0;" ::"r"(CW * 32) : "memory");
    }
    // ldsm_x4 weight loads and the matching x reads whenever a chunk lies in
    // one scale group (always for scale-after): free of bank conflicts
    const bool tx = SA || gshift >= 7;
    uint32_t xaddr[NT];
    bool xon[NT];
    const XT *xg[NT];
#pragma unroll
    for (int j = 0; j < NT; ++j) {
        const int mb = 8 * j + gi;
        xon[j] = mb < m;
        const int mr = xon[j] ? mb : 0;
        xaddr[j] = smem_u32(xs) + (uint32_t)(mr * xstride + (tx ? 8 : 32) * t) * 2u;  // tx: ldsm_x4 layout
        xg[j] = x + (size_t)mr * k + (tx ? 8 : 32) * t;
    }
    uint4 xb[NT];
#pragma unroll
    for (int j = 0; j < NT; ++j) xb[j] = make_uint4(0, 0, 0, 0);
    float acc[2][NT][4];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int j = 0; j < NT; ++j) acc[a][j][0] = acc[a][j][1] = acc[a][j][2] = acc[a][j][3] = 0.0f;

    bool ok = true;
    float gsave = 0.0f;  // SiLU-gate mode: this thread's reduced gate value
    int ti = 0, st = 0;
    for (int pos = 0; pos < npos; ++pos) {
        const int slot = pos % nstages, round = pos / nstages;
        const int row0 = tile_row0(ti);
        // Scales without TMA: each lane reads its two rows' scales for its
        // chunks of this stage straight from global memory.
        float sreg[CPW][2];
        if (!STMA) {
            const int ra = min(row0 + gi, n - 1), rb = min(row0 + gi + 8, n - 1);
#pragma unroll
            for (int q = 0; q < CPW; ++q) {
                const int c = st * CW * CPW + warp + q * CW;
                const int col = min((128 * c + 32 * t) >> gshift, groups - 1);
                sreg[q][0] = load_scale(scales, (size_t)ra * groups + col, half_scales);
                sreg[q][1] = load_scale(scales, (size_t)rb * groups + col, half_scales);
            }
        }
        // warp-uniform: ldmatrix and mma.sync below are warp-collective
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&full[slot], round & 1));
        if (ok) {
            const uint8_t *wst = wbuf + (size_t)slot * L::kStageBytes;
            const float *sst = reinterpret_cast<const float *>(reinterpret_cast<const uint8_t *>(sbuf) + (size_t)slot * sbytes);
            auto do_chunk = [&](int q) {
                const int cs = warp + q * CW;            // chunk within the stage
                const int c = st * CW * CPW + cs;        // chunk within the row
                // Chunk cs = 64 bytes of each row: box cs/2, chunk
                // ((cs%2)*4 + t) of the 128-byte row, swizzled by row % 8.
                uint32_t qa[4], qb[4];
                if (tx) {  // warp-uniform
                    const int lr = lane & 7, lj = lane >> 3;  // ldmatrix row / matrix of this lane
                    const uint32_t a = smem_u32(wst) + (uint32_t)(cs >> 1) * 2048u + (uint32_t)lr * 128u +
                                       (uint32_t)(((((cs & 1) << 2) + lj) ^ lr) << 4);
                    ldsm_x4(a, qa);
                    ldsm_x4(a + 8u * 128u, qb);
                } else {
                    const uint32_t piece = (uint32_t)(cs >> 1) * 2048u + (uint32_t)gi * 128u +
                                           (uint32_t)(((((cs & 1) << 2) + t) ^ (gi & 7)) << 4);
                    const uint4 wa = *reinterpret_cast<const uint4 *>(wst + piece);
                    const uint4 wb = *reinterpret_cast<const uint4 *>(wst + piece + 8 * 128);
                    qa[0] = wa.x, qa[1] = wa.y, qa[2] = wa.z, qa[3] = wa.w;
                    qb[0] = wb.x, qb[1] = wb.y, qb[2] = wb.z, qb[3] = wb.w;
                }
                const int scol = (cs * 128 + 32 * t) >> gshift;
                float sa, sb;
                if (STMA && half_scales) {  // fp16 scale box: 16 rows of spr halves, unswizzled
                    const __half *sh = reinterpret_cast<const __half *>(sst);
                    sa = __half2float(sh[gi * spr + scol]);
                    sb = __half2float(sh[(gi + 8) * spr + scol]);
                } else if (STMA) {
                    stage_scales(sst, gi, scol, spr, sa, sb);
                } else {
                    sa = sreg[q][0], sb = sreg[q][1];
                }
                const bool in = 128 * c + 32 * t < kp;
                if constexpr (SA) {
                    gemv_chunk_sa<NT, XS, FOLD, true>(c, qa, qb, in ? sa : 0.0f, in ? sb : 0.0f, xaddr, xon, xg, xb, acc,
                                                corr + c * 16 + 2 * t);
                } else {
                    const DqScale dsa = make_dq_scale(in ? sa : 0.0f), dsb = make_dq_scale(in ? sb : 0.0f);
                    if (__all_sync(0xffffffffu, dsa.fast && dsb.fast))
                        gemv_chunk<XT, NT, XS, true>(c, qa, qb, dsa, dsb, xaddr, xon, xg, xb, acc, tx ? 32 : 8);
                    else
                        gemv_chunk<XT, NT, XS, false>(c, qa, qb, dsa, dsb, xaddr, xon, xg, xb, acc, tx ? 32 : 8);
                }
            };
            if (st * CW * CPW + (CPW - 1) * CW + warp < nchunks) {
                // Every chunk of this warp is inside K: no per-chunk branch,
                // so the chunks' instruction streams can interleave.
#pragma unroll
                for (int q = 0; q < CPW; ++q) do_chunk(q);
            } else {
#pragma unroll
                for (int q = 0; q < CPW; ++q)
                    if (st * CW * CPW + warp + q * CW < nchunks) do_chunk(q);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        if (++st == spt) {
            const int buf = nred == 2 ? (ti & 1) : 0;
#pragma unroll
            for (int j = 0; j < NT; ++j)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    red[buf][warp][j][e][lane] = acc[0][j][e] + acc[1][j][e];
                    acc[0][j][e] = 0.0f;
                    acc[1][j][e] = 0.0f;
                }
            asm volatile("bar.sync 1, %0;" ::"r"(CW * 32) : "memory");
            for (int idx = threadIdx.x; idx < NT * 4 * 32; idx += CW * 32) {
                const int j = idx / 128, e = (idx / 32) % 4, ln = idx % 32;
                float v = 0.0f;
#pragma unroll
                for (int wv = 0; wv < CW; ++wv) v += red[buf][wv][j][e][ln];
                const int g2 = ln >> 2, t2 = ln & 3;
                const int row = row0 + g2 + (e >= 2 ? 8 : 0);
                const int mb = 8 * j + 2 * t2 + (e & 1);
                if (gate_n == 0) {
                    if (ok && row < n && mb < m) y.store(mb, row, v);
                } else if ((ti & 1) == 0) {
                    gsave = v;  // gate tile: kept until the matching up tile
                } else {
                    const int f = row - gate_n;  // output feature
                    if (ok && f < gate_n && mb < m) y.store(mb, f, gsave / (1.0f + expf(-gsave)) * v);
                }
            }
            // One reduction slot: every read of it ends before the next
            // tile's partial sums are written.
            if (nred == 1) asm volatile("bar.sync 1, %0;" ::"r"(CW * 32) : "memory");
            st = 0;
            ++ti;
        }
    }
}

// ----------------------------------------------------------- tile GEMV ----
//
// Small decode layers (KP <= 4096, one 16-row tile per CTA): 8 warps and no
// producer warp, up to four CTAs per SM -- two of this launch and two of the
// next, which then streams its tile (static weights) while this one
// computes.  Thread 0 issues the tile's TMA boxes (the 32 KB stage and the
// scale box of gemv_tma_kernel) at entry; after griddepcontrol.wait every
// warp takes chunks w, w + 8, ... exactly as gemv_tma_kernel's consumers do
// and the partial sums are reduced in the same fixed order, so both kernels
// give identical results.
template <typename XT, int NT, bool SA, bool XS, bool STMA>
__global__ void __launch_bounds__(256, 4)
    gemv_tile_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap smap,
                     const XT *__restrict__ x, const float *__restrict__ scales, OutSpec y, int m, int n,
                     int k, int kp, int gshift, int xstride, int prefetch) {
    static_assert(!SA || std::is_same<XT, __half>::value, "scale-after mode is for fp16 x");
    constexpr int CW = 8, CPW = 4;
    using L = TmaGemvLayout<CW, CPW>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    const int spr = L::kStageCols >> gshift;  // scales per row in the stage
    const int sbytes = ((16 * spr * 4 + 127) / 128) * 128;
    const uint8_t *wst = smem;                                               // [boxes][16][128]
    float *sst = reinterpret_cast<float *>(smem + L::kStageBytes);           // [16][spr]
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::kStageBytes + sbytes);
    auto red = reinterpret_cast<float(*)[NT][4][32]>(full + 2);              // [CW]
    XT *xs = reinterpret_cast<XT *>(reinterpret_cast<uint8_t *>(red) + gemv_red_bytes(CW, NT) / 2);
    constexpr bool FOLD = SA && XS;  // bias-folded dequantization (gemv_chunk_sa)
    float *corr = reinterpret_cast<float *>(xs + (size_t)m * xstride);  // [chunks][16]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gi = lane >> 2, t = lane & 3;
    const int groups = kp >> gshift;
    const int nchunks = (kp + 127) >> 7;
    const int row0 = (int)blockIdx.x * 16;

    // Dependent launches may start now; they wait for this grid before
    // touching anything it writes.
    asm volatile("griddepcontrol.launch_dependents;");
    if (threadIdx.x == 0) {
        mbar_init(&full[0], 1);
        fence_barrier_init();
        tma_prefetch_desc(&wmap);
        if (STMA) tma_prefetch_desc(&smap);
        if (!prefetch) asm volatile("griddepcontrol.wait;" ::: "memory");
        mbar_arrive_expect_tx(&full[0], L::kStageBytes + (STMA ? 16 * spr * 4 : 0));
#pragma unroll
        for (int b = 0; b < L::kBoxes; ++b)
            tma_load_2d(smem + b * 2048, &wmap, &full[0], 128 * b, row0);
        if (STMA) tma_load_2d(sst, &smap, &full[0], 0, row0);
    }

    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (XS) gemv_stage_x<XT, SA, FOLD>(x, xs, corr, m, k, kp, xstride, CW * 32);
    __syncthreads();  // xs staged; full[0] initialised before anyone waits on it
    // ldsm_x4 weight loads and the matching x reads whenever a chunk lies in
    // one scale group (always for scale-after): free of bank conflicts
    const bool tx = SA || gshift >= 7;
    uint32_t xaddr[NT];
    bool xon[NT];
    const XT *xg[NT];
#pragma unroll
    for (int j = 0; j < NT; ++j) {
        const int mb = 8 * j + gi;
        xon[j] = mb < m;
        const int mr = xon[j] ? mb : 0;
        xaddr[j] = smem_u32(xs) + (uint32_t)(mr * xstride + (tx ? 8 : 32) * t) * 2u;  // tx: ldsm_x4 layout
        xg[j] = x + (size_t)mr * k + (tx ? 8 : 32) * t;
    }
    uint4 xb[NT];
#pragma unroll
    for (int j = 0; j < NT; ++j) xb[j] = make_uint4(0, 0, 0, 0);
    float acc[2][NT][4];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int j = 0; j < NT; ++j) acc[a][j][0] = acc[a][j][1] = acc[a][j][2] = acc[a][j][3] = 0.0f;

    float sreg[CPW][2];
    if (!STMA) {  // scales straight from global memory (row pitch not 16-byte aligned)
        const int ra = min(row0 + gi, n - 1), rb = min(row0 + gi + 8, n - 1);
#pragma unroll
        for (int q = 0; q < CPW; ++q) {
            const int c = warp + q * CW;
            const int col = min((128 * c + 32 * t) >> gshift, groups - 1);
            sreg[q][0] = __ldg(scales + (size_t)ra * groups + col);
            sreg[q][1] = __ldg(scales + (size_t)rb * groups + col);
        }
    }
    const bool ok = __all_sync(0xffffffffu, mbar_wait(&full[0], 0));  // warp-uniform, as above
    if (ok) {
        auto do_chunk = [&](int q) {
            const int c = warp + q * CW;  // chunk within the row (the stage is the whole row)
            uint32_t qa[4], qb[4];
            if (tx) {  // warp-uniform
                const int lr = lane & 7, lj = lane >> 3;  // ldmatrix row / matrix of this lane
                const uint32_t a = smem_u32(wst) + (uint32_t)(c >> 1) * 2048u + (uint32_t)lr * 128u +
                                   (uint32_t)(((((c & 1) << 2) + lj) ^ lr) << 4);
                ldsm_x4(a, qa);
                ldsm_x4(a + 8u * 128u, qb);
            } else {
                const uint32_t piece = (uint32_t)(c >> 1) * 2048u + (uint32_t)gi * 128u +
                                       (uint32_t)(((((c & 1) << 2) + t) ^ (gi & 7)) << 4);
                const uint4 wa = *reinterpret_cast<const uint4 *>(wst + piece);
                const uint4 wb = *reinterpret_cast<const uint4 *>(wst + piece + 8 * 128);
                qa[0] = wa.x, qa[1] = wa.y, qa[2] = wa.z, qa[3] = wa.w;
                qb[0] = wb.x, qb[1] = wb.y, qb[2] = wb.z, qb[3] = wb.w;
            }
            const int scol = (c * 128 + 32 * t) >> gshift;
            float sa, sb;
            if (STMA)
                stage_scales(sst, gi, scol, spr, sa, sb);
            else
                sa = sreg[q][0], sb = sreg[q][1];
            const bool in = 128 * c + 32 * t < kp;
            if constexpr (SA) {
                gemv_chunk_sa<NT, XS, FOLD, true>(c, qa, qb, in ? sa : 0.0f, in ? sb : 0.0f, xaddr, xon, xg, xb, acc,
                                            corr + c * 16 + 2 * t);
            } else {
                const DqScale dsa = make_dq_scale(in ? sa : 0.0f), dsb = make_dq_scale(in ? sb : 0.0f);
                if (__all_sync(0xffffffffu, dsa.fast && dsb.fast))
                    gemv_chunk<XT, NT, XS, true>(c, qa, qb, dsa, dsb, xaddr, xon, xg, xb, acc, tx ? 32 : 8);
                else
                    gemv_chunk<XT, NT, XS, false>(c, qa, qb, dsa, dsb, xaddr, xon, xg, xb, acc, tx ? 32 : 8);
            }
        };
        if ((CPW - 1) * CW + warp < nchunks) {
#pragma unroll
            for (int q = 0; q < CPW; ++q) do_chunk(q);
        } else {
#pragma unroll
            for (int q = 0; q < CPW; ++q)
                if (warp + q * CW < nchunks) do_chunk(q);
        }
    }
    // Fixed-order reduction over the warps, as in gemv_tma_kernel.
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) red[warp][j][e][lane] = acc[0][j][e] + acc[1][j][e];
    __syncthreads();
    for (int idx = threadIdx.x; idx < NT * 4 * 32; idx += CW * 32) {
        const int j = idx / 128, e = (idx / 32) % 4, ln = idx % 32;
        float v = 0.0f;
#pragma unroll
        for (int wv = 0; wv < CW; ++wv) v += red[wv][j][e][ln];
        const int g2 = ln >> 2, t2 = ln & 3;
        const int row = row0 + g2 + (e >= 2 ? 8 : 0);
        const int mb = 8 * j + 2 * t2 + (e & 1);
        if (ok && row < n && mb < m) y.store(mb, row, v);
    }
}

// ----------------------------------------------------------- pair GEMV ----
//
// Small decode layers (KP <= 4096, at most two 16-row tiles per SM): one CTA
// per SM, 16 warps, at most 64 registers, so exactly two CTAs fit on an SM.
// In back-to-back launches every SM then holds one CTA of the previous launch
// and receives exactly one of this one -- the placement stays balanced --
// and this launch's weights (static) stream while the previous one finishes.
// The CTA owns tiles blockIdx.x and blockIdx.x + gridDim.x; thread 0 issues
// both tiles' TMA boxes at entry, and after griddepcontrol.wait warps 0-7
// compute the first tile while warps 8-15 compute the second, each group with
// gemv_tma_kernel's chunk -> warp map and fixed-order reduction (identical
// results).
template <typename XT, int NT, bool SA, bool XS, bool STMA>
__global__ void __launch_bounds__(512, 2)
    gemv_pair_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap smap,
                     const XT *__restrict__ x, const float *__restrict__ scales, OutSpec y, int m, int n,
                     int k, int kp, int gshift, int xstride, int prefetch, int half_scales) {
    static_assert(!SA || std::is_same<XT, __half>::value, "scale-after mode is for fp16 x");
    constexpr int CW = 8, CPW = 4;
    using L = TmaGemvLayout<CW, CPW>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    const int spr = L::kStageCols >> gshift;  // scales per row in a stage
    const int sbytes = ((16 * spr * 4 + 127) / 128) * 128;
    const int stage_bytes = L::kStageBytes + sbytes;                      // a multiple of 1024 + 128 k
    const int stage_pitch = (stage_bytes + 1023) / 1024 * 1024;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + 2 * stage_pitch);
    auto red = reinterpret_cast<float(*)[CW][NT][4][32]>(full + 2);      // [2 groups]
    XT *xs = reinterpret_cast<XT *>(reinterpret_cast<uint8_t *>(red) + gemv_red_bytes(CW, NT));
    constexpr bool FOLD = SA && XS;  // bias-folded dequantization (gemv_chunk_sa)
    float *corr = reinterpret_cast<float *>(xs + (size_t)m * xstride);  // [chunks][16]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int grp = warp >> 3, wg = warp & 7;
    const int gi = lane >> 2, t = lane & 3;
    const int groups = kp >> gshift;
    const int nchunks = (kp + 127) >> 7;
    const int tiles = (n + 15) >> 4;
    const int ntiles = (int)blockIdx.x + (int)gridDim.x < tiles ? 2 : 1;

    asm volatile("griddepcontrol.launch_dependents;");
    if (threadIdx.x == 0) {
        mbar_init(&full[0], 1);
        mbar_init(&full[1], 1);
        fence_barrier_init();
        tma_prefetch_desc(&wmap);
        if (STMA) tma_prefetch_desc(&smap);
        if (!prefetch) asm volatile("griddepcontrol.wait;" ::: "memory");
        for (int tt = 0; tt < ntiles; ++tt) {
            uint8_t *st = smem + tt * stage_pitch;
            const int r0 = ((int)blockIdx.x + tt * (int)gridDim.x) * 16;
            mbar_arrive_expect_tx(&full[tt], L::kStageBytes + (STMA ? 16 * spr * (half_scales ? 2 : 4) : 0));
#pragma unroll
            for (int b = 0; b < L::kBoxes; ++b) tma_load_2d(st + b * 2048, &wmap, &full[tt], 128 * b, r0);
            if (STMA) tma_load_2d(st + L::kStageBytes, &smap, &full[tt], 0, r0);
        }
    }

    __syncthreads();  // the barriers initialised before anyone waits on them
    if (grp >= ntiles) return;  // no second tile: the second warp group is done
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // Each warp stages the x its own chunks read: no CTA-wide barrier after the wait.
    if (XS) gemv_stage_x_warp<XT, SA, FOLD, 2 * NT>(x, xs, corr, m, k, xstride, wg, lane, nchunks);
    __syncwarp();

    const uint8_t *wst = smem + grp * stage_pitch;
    const float *sst = reinterpret_cast<const float *>(wst + L::kStageBytes);
    const int row0 = ((int)blockIdx.x + grp * (int)gridDim.x) * 16;
    // ldsm_x4 weight loads and the matching x reads whenever a chunk lies in
    // one scale group (always for scale-after): free of bank conflicts
    const bool tx = SA || gshift >= 7;
    uint32_t xaddr[NT];
    bool xon[NT];
    const XT *xg[NT];
#pragma unroll
    for (int j = 0; j < NT; ++j) {
        const int mb = 8 * j + gi;
        xon[j] = mb < m;
        const int mr = xon[j] ? mb : 0;
        xaddr[j] = smem_u32(xs) + (uint32_t)(mr * xstride + (tx ? 8 : 32) * t) * 2u;  // tx: ldsm_x4 layout
        xg[j] = x + (size_t)mr * k + (tx ? 8 : 32) * t;
    }
    uint4 xb[NT];
#pragma unroll
    for (int j = 0; j < NT; ++j) xb[j] = make_uint4(0, 0, 0, 0);
    float acc[2][NT][4];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int j = 0; j < NT; ++j) acc[a][j][0] = acc[a][j][1] = acc[a][j][2] = acc[a][j][3] = 0.0f;

    float sreg[CPW][2];
    if (!STMA) {  // scales straight from global memory (row pitch not 16-byte aligned)
        const int ra = min(row0 + gi, n - 1), rb = min(row0 + gi + 8, n - 1);
#pragma unroll
        for (int q = 0; q < CPW; ++q) {
            const int c = wg + q * CW;
            const int col = min((128 * c + 32 * t) >> gshift, groups - 1);
            sreg[q][0] = load_scale(scales, (size_t)ra * groups + col, half_scales);
            sreg[q][1] = load_scale(scales, (size_t)rb * groups + col, half_scales);
        }
    }
    const bool ok = __all_sync(0xffffffffu, mbar_wait(&full[grp], 0));  // warp-uniform, as above
    if (ok) {
        auto do_chunk = [&](int q) {
            const int c = wg + q * CW;
            uint32_t qa[4], qb[4];
            if (tx) {  // warp-uniform
                const int lr = lane & 7, lj = lane >> 3;  // ldmatrix row / matrix of this lane
                const uint32_t a = smem_u32(wst) + (uint32_t)(c >> 1) * 2048u + (uint32_t)lr * 128u +
                                   (uint32_t)(((((c & 1) << 2) + lj) ^ lr) << 4);
                ldsm_x4(a, qa);
                ldsm_x4(a + 8u * 128u, qb);
            } else {
                const uint32_t piece = (uint32_t)(c >> 1) * 2048u + (uint32_t)gi * 128u +
                                       (uint32_t)(((((c & 1) << 2) + t) ^ (gi & 7)) << 4);
                const uint4 wa = *reinterpret_cast<const uint4 *>(wst + piece);
                const uint4 wb = *reinterpret_cast<const uint4 *>(wst + piece + 8 * 128);
                qa[0] = wa.x, qa[1] = wa.y, qa[2] = wa.z, qa[3] = wa.w;
                qb[0] = wb.x, qb[1] = wb.y, qb[2] = wb.z, qb[3] = wb.w;
            }
            const int scol = (c * 128 + 32 * t) >> gshift;
            float sa, sb;
            if (STMA && half_scales) {  // fp16 scale box: 16 rows of spr halves, unswizzled
                const __half *sh = reinterpret_cast<const __half *>(sst);
                sa = __half2float(sh[gi * spr + scol]);
                sb = __half2float(sh[(gi + 8) * spr + scol]);
            } else if (STMA) {
                stage_scales(sst, gi, scol, spr, sa, sb);
            } else {
                sa = sreg[q][0], sb = sreg[q][1];
            }
            const bool in = 128 * c + 32 * t < kp;
            if constexpr (SA) {
                gemv_chunk_sa<NT, XS, FOLD, true>(c, qa, qb, in ? sa : 0.0f, in ? sb : 0.0f, xaddr, xon, xg, xb, acc,
                                            corr + c * 16 + 2 * t);
            } else {
                const DqScale dsa = make_dq_scale(in ? sa : 0.0f), dsb = make_dq_scale(in ? sb : 0.0f);
                if (__all_sync(0xffffffffu, dsa.fast && dsb.fast))
                    gemv_chunk<XT, NT, XS, true>(c, qa, qb, dsa, dsb, xaddr, xon, xg, xb, acc, tx ? 32 : 8);
                else
                    gemv_chunk<XT, NT, XS, false>(c, qa, qb, dsa, dsb, xaddr, xon, xg, xb, acc, tx ? 32 : 8);
            }
        };
        if ((CPW - 1) * CW + wg < nchunks) {
#pragma unroll
            for (int q = 0; q < CPW; ++q) do_chunk(q);
        } else {
#pragma unroll
            for (int q = 0; q < CPW; ++q)
                if (wg + q * CW < nchunks) do_chunk(q);
        }
    }
    // Fixed-order reduction over the group's 8 warps (named barrier per group).
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) red[grp][wg][j][e][lane] = acc[0][j][e] + acc[1][j][e];
    asm volatile("bar.sync %0, 256;" ::"r"(1 + grp) : "memory");
    for (int idx = threadIdx.x & 255; idx < NT * 4 * 32; idx += 256) {
        const int j = idx / 128, e = (idx / 32) % 4, ln = idx % 32;
        float v = 0.0f;
#pragma unroll
        for (int wv = 0; wv < CW; ++wv) v += red[grp][wv][j][e][ln];
        const int g2 = ln >> 2, t2 = ln & 3;
        const int row = row0 + g2 + (e >= 2 ? 8 : 0);
        const int mb = 8 * j + 2 * t2 + (e & 1);
        if (ok && row < n && mb < m) y.store(mb, row, v);
    }
}

// ------------------------------------------------------------- SIMT ----
//
// Any shape and any even group size: one warp per weight row, lanes stride
// over K, up to 8 batch rows per pass (more passes for larger M).
template <typename XT>
__global__ void __launch_bounds__(256) simt_int4_kernel(const XT *__restrict__ x, const uint8_t *__restrict__ packed,
                                                        const float *__restrict__ scales, OutSpec y,
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
                if (lane == 0 && m0 + i < m) y.store(m0 + i, (int)row, v);
            }
        }
    }
}

// Shared memory per block (opt-in maximum), cached per device.
inline int max_smem_optin() {
    static int cached[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 227 * 1024;
    if (cached[dev] == 0) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess || v <= 0)
            v = 227 * 1024;
        cached[dev] = v;
    }
    return cached[dev];
}

// Opts a kernel into the device's maximum dynamic shared memory, once per
// (kernel, device).
inline int allow_max_smem(const void *kern) {
    static std::mutex mu;
    static std::set<std::pair<const void *, int>> done;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    if (done.count({kern, dev})) return OQ_OK;
    OQ_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem_optin()));
    done.insert({kern, dev});
    return OQ_OK;
}

// Launch with programmatic stream serialization: a GEMV that follows a
// PDL-triggering kernel in the stream may start while that kernel drains
// (and, with `prefetch`, stream its static weights meanwhile).  After any
// other kernel it behaves like a normal launch.
template <typename Kern, typename XT>
int launch_pdl(Kern kern, unsigned blocks, unsigned threads, size_t smem, cudaStream_t st, const XT *x,
               const uint8_t *packed, const float *scales, OutSpec y, int m, int n, int k, int kp, int gshift,
               int xstride, int prefetch) {
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
    cudaError_t err = cudaLaunchKernelEx(&cfg, kern, x, packed, scales, y, m, n, k, kp, gshift, xstride, prefetch);
    if (err != cudaSuccess) {
        set_error("int4_linear (GEMV): launch failed: %s", cudaGetErrorString(err));
        return OQ_ERR_CUDA;
    }
    return OQ_OK;
}

constexpr size_t kGemvMaxXs = 96 * 1024;  // staged-x limit (two CTAs per SM)

// Bytes of x staged in shared memory (0 = x read from global memory).
inline size_t gemv_xs_bytes(int64_t m, int64_t kp, int xsize) {
    const int64_t xstride = cdiv(kp, 128) * 128 + 8;
    const size_t b = (size_t)(m * xstride * xsize);
    return b <= kGemvMaxXs ? b : 0;
}

template <typename XT, int NT, int WARPS, int U, int MINB, bool SA>
int launch_gemv_t(const XT *x, const uint8_t *packed, const float *scales, OutSpec y, int64_t m, int64_t n,
                  int64_t k, int64_t kp, int gshift, int prefetch, cudaStream_t st) {
    // Persistent grid: MINB CTAs per SM, each looping over 16-row tiles.
    const int64_t tiles = cdiv(n, 16);
    const unsigned blocks = (unsigned)std::min<int64_t>(tiles, (int64_t)sm_count() * MINB);
    const int xstride = (int)(cdiv(kp, 128) * 128 + 8);
    const size_t xbytes = gemv_xs_bytes(m, kp, (int)sizeof(XT));
    const size_t smem = gemv_red_bytes(WARPS, NT) + xbytes;
    auto kern = xbytes ? gemv_int4_kernel<XT, NT, WARPS, U, true, MINB, SA>
                       : gemv_int4_kernel<XT, NT, WARPS, U, false, MINB, SA>;
    const int rc = allow_max_smem(reinterpret_cast<const void *>(kern));
    if (rc != OQ_OK) return rc;
    return launch_pdl(kern, blocks, WARPS * 32, smem, st, x, packed, scales, y, (int)m, (int)n, (int)k, (int)kp,
                      gshift, xstride, prefetch);
}

// Stage count and shared-memory bytes of the TMA GEMV, or 0 stages when the
// shape does not fit.  x (and, for the scale-after path, its bias table:
// gemv_stage_x) is staged in shared memory whenever two stages still fit
// (*xs_out = 1): reading x from global memory in every chunk costs more than
// further stages hide.  To make room for a large x (M = 16) the cross-warp
// reduction buffer drops from two tile slots to one (*nred_out = 1; the
// kernel then takes one more barrier per tile).  Without staged x the stages
// must be whole (KP a multiple of the stage width and K == KP).
template <int CW, int CPW>
inline int tma_gemv_plan(int64_t m, int64_t k, int64_t kp, int g, int nt, int xsize, size_t *smem_out,
                         int *xstride_out, bool *xs_out, int *nred_out, int ctas_per_sm = 1,
                         int64_t max_pos = 1 << 30) {
    using L = TmaGemvLayout<CW, CPW>;
    if (g < 32 || g > L::kStageCols) return 0;
    const int64_t xstride = cdiv(kp, 128) * 128 + gemv_xpad(g);  // chunks past KP are skipped
    const int64_t spr = L::kStageCols / g;
    const size_t sbytes = (size_t)cdiv(16 * spr * 4, 128) * 128;
    const size_t per_stage = (size_t)L::kStageBytes + sbytes + 16;
    const size_t cap = (size_t)max_smem_optin() / ctas_per_sm - (ctas_per_sm > 1 ? 1024 : 0);
    const size_t red2 = gemv_red_bytes(CW, nt);  // two tile slots
    const size_t xbytes = (size_t)(m * xstride * xsize) + (size_t)cdiv(kp, 128) * 16 * 4;
    int nred = 2;
    bool xs = 1024 + red2 + xbytes + 2 * per_stage <= cap;
    if (!xs && 1024 + red2 / 2 + xbytes + 2 * per_stage <= cap) xs = true, nred = 1;
    if (!xs && !(kp == k && kp % L::kStageCols == 0)) return 0;
    const size_t fixed = 1024 + red2 / 2 * nred + (xs ? xbytes : 0);
    if (fixed + 2 * per_stage > cap) return 0;
    int stages = (int)std::min<size_t>(8, (cap - fixed) / per_stage);
    stages = (int)std::max<int64_t>(2, std::min<int64_t>(stages, max_pos));
    *smem_out = fixed + stages * per_stage;
    *xstride_out = (int)xstride;
    *xs_out = xs;
    *nred_out = nred;
    return stages;
}

// Tensor maps of the TMA GEMVs: the packed rows in 16-row x 128-byte boxes
// (128-byte swizzle) and, when the scale row pitch is a multiple of 16 bytes,
// the scales in 16-row boxes of one stage's groups (*stma = true).
template <int CW, int CPW>
int make_gemv_maps(const uint8_t *packed, const float *scales, int64_t n, int64_t kp, int g, CUtensorMap *wmap,
                   CUtensorMap *smap, bool *stma) {
    using L = TmaGemvLayout<CW, CPW>;
    int rc = make_tensor_map_2d(wmap, packed, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)(kp / 2), (uint64_t)n,
                                (uint64_t)(kp / 2), 128, 16, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != OQ_OK) return rc;
    const int64_t groups = kp / g;
    *stma = (groups * 4) % 16 == 0 && aligned(scales, 16) && (L::kStageCols / g) * 4 % 16 == 0;
    if (*stma) {
        rc = make_tensor_map_2d(smap, scales, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)groups, (uint64_t)n,
                                (uint64_t)(groups * 4), (uint32_t)(L::kStageCols / g), 16,
                                (L::kStageCols / g) * 4 == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                                                 : CU_TENSOR_MAP_SWIZZLE_NONE);  // see stage_scales
        if (rc != OQ_OK) return rc;
    } else {
        *smap = *wmap;  // unused
    }
    return OQ_OK;
}

template <typename XT, int NT, int CW, int CPW, bool SA, int CTAS = 1>
int launch_gemv_tma(const XT *x, const uint8_t *packed, const float *scales, OutSpec y, int64_t m, int64_t n,
                    int64_t k, int64_t kp, int g, int gshift, int prefetch, cudaStream_t st, int64_t gate_n = 0,
                    bool half_scales = false) {
    using L = TmaGemvLayout<CW, CPW>;
    size_t smem = 0;
    int xstride = 0;
    bool xs = false;
    // units: 16-row tiles, or (gate_n > 0) gate/up tile pairs
    const int64_t units = gate_n ? cdiv(gate_n, 16) : cdiv(n, 16);
    const int64_t grid = std::min<int64_t>(units, (int64_t)sm_count() * CTAS);
    const int64_t max_pos = cdiv(units, grid) * (gate_n ? 2 : 1) * cdiv(kp, L::kStageCols);
    int nred = 2;
    const int stages =
        tma_gemv_plan<CW, CPW>(m, k, kp, g, NT, (int)sizeof(XT), &smem, &xstride, &xs, &nred, CTAS, max_pos);
    if (stages == 0) return invalid("TMA GEMV: shape does not fit in shared memory");
    CUtensorMap wmap, smap;
    bool stma = false;
    int rc = make_gemv_maps<CW, CPW>(packed, scales, n, kp, g, &wmap, &smap, &stma);
    if (rc != OQ_OK) return rc;
    if (half_scales) {
        // fp16 scales by TMA too: a box of the stage's groups x 16 rows
        // (2-byte elements, rows of groups * 2 bytes), read unswizzled
        const int64_t groups = kp / g, spr = L::kStageCols / g;
        stma = (groups * 2) % 16 == 0 && (spr * 2) % 16 == 0 && aligned(scales, 16);
        if (stma) {
            rc = make_tensor_map_2d(&smap, scales, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)groups, (uint64_t)n,
                                    (uint64_t)(groups * 2), (uint32_t)spr, 16, CU_TENSOR_MAP_SWIZZLE_NONE);
            if (rc != OQ_OK) return rc;
        }
    }
    auto pick = [&](auto kern) -> int {
        int rc2 = allow_max_smem(reinterpret_cast<const void *>(kern));
        if (rc2 != OQ_OK) return rc2;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)grid);
        cfg.blockDim = dim3((CW + 1) * 32);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        cudaError_t err = cudaLaunchKernelEx(&cfg, kern, wmap, smap, x, scales, y, (int)m, (int)n, (int)k, (int)kp,
                                             gshift, xstride, stages, prefetch, (int)gate_n, nred,
                                             half_scales ? 1 : 0);
        if (err != cudaSuccess) {
            set_error("int4_linear (TMA GEMV): launch failed: %s", cudaGetErrorString(err));
            return OQ_ERR_CUDA;
        }
        return OQ_OK;
    };
    if (xs)
        return stma ? pick(gemv_tma_kernel<XT, NT, CW, CPW, SA, true, true>)
                    : pick(gemv_tma_kernel<XT, NT, CW, CPW, SA, true, false>);
    return stma ? pick(gemv_tma_kernel<XT, NT, CW, CPW, SA, false, true>)
                : pick(gemv_tma_kernel<XT, NT, CW, CPW, SA, false, false>);
}

// Tile GEMV (config 12): x staged in shared memory up to this size, else read
// from global memory (needs KP == K, whole 128-column chunks).
constexpr int64_t kTileXs = 16 * 1024;

inline bool gemv_tile_ok(int64_t m, int64_t n, int64_t k, int64_t kp, int g, const uint8_t *packed) {
    const int64_t xstride = cdiv(kp, 128) * 128 + gemv_xpad(g);
    const bool xs = m * xstride * 2 <= kTileXs;
    return m <= 16 && g >= 32 && g <= 4096 && kp <= 4096 && aligned(packed, 16) && (kp / 2) % 16 == 0 &&
           n < (1ll << 31) && (xs || (kp == k && kp % 128 == 0));
}

template <typename XT, int NT, bool SA>
int launch_gemv_tile(const XT *x, const uint8_t *packed, const float *scales, OutSpec y, int64_t m, int64_t n,
                     int64_t k, int64_t kp, int g, int gshift, int prefetch, cudaStream_t st) {
    using L = TmaGemvLayout<8, 4>;
    if (!gemv_tile_ok(m, n, k, kp, g, packed)) return invalid("tile GEMV (config 12) does not take this shape");
    const int64_t xstride = cdiv(kp, 128) * 128 + gemv_xpad(g);
    const size_t xbytes = (size_t)(m * xstride) * sizeof(XT);
    const bool xs = (int64_t)xbytes <= kTileXs;
    const size_t sbytes = (size_t)cdiv(16 * (L::kStageCols / g) * 4, 128) * 128;
    const size_t cbytes = (SA && xs) ? (size_t)cdiv(kp, 128) * 16 * 4 : 0;  // bias table
    const size_t smem = 1024 + L::kStageBytes + sbytes + 16 + gemv_red_bytes(8, NT) / 2 + (xs ? xbytes : 0) + cbytes;
    CUtensorMap wmap, smap;
    bool stma = false;
    int rc = make_gemv_maps<8, 4>(packed, scales, n, kp, g, &wmap, &smap, &stma);
    if (rc != OQ_OK) return rc;
    auto pick = [&](auto kern) -> int {
        int rc2 = allow_dynamic_smem(reinterpret_cast<const void *>(kern), smem);
        if (rc2 != OQ_OK) return rc2;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)cdiv(n, 16));
        cfg.blockDim = dim3(256);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        cudaError_t err = cudaLaunchKernelEx(&cfg, kern, wmap, smap, x, scales, y, (int)m, (int)n, (int)k, (int)kp,
                                             gshift, (int)xstride, prefetch);
        if (err != cudaSuccess) {
            set_error("int4_linear (tile GEMV): launch failed: %s", cudaGetErrorString(err));
            return OQ_ERR_CUDA;
        }
        return OQ_OK;
    };
    if (xs)
        return stma ? pick(gemv_tile_kernel<XT, NT, SA, true, true>) : pick(gemv_tile_kernel<XT, NT, SA, true, false>);
    return stma ? pick(gemv_tile_kernel<XT, NT, SA, false, true>) : pick(gemv_tile_kernel<XT, NT, SA, false, false>);
}

// Pair GEMV (config 13): the tile GEMV's shapes with at most two tiles per SM.
inline bool gemv_pair_ok(int64_t m, int64_t n, int64_t k, int64_t kp, int g, const uint8_t *packed) {
    return gemv_tile_ok(m, n, k, kp, g, packed) && cdiv(n, 16) <= 2 * (int64_t)sm_count();
}

template <typename XT, int NT, bool SA>
int launch_gemv_pair(const XT *x, const uint8_t *packed, const float *scales, OutSpec y, int64_t m, int64_t n,
                     int64_t k, int64_t kp, int g, int gshift, int prefetch, cudaStream_t st,
                     bool half_scales = false) {
    using L = TmaGemvLayout<8, 4>;
    if (!gemv_pair_ok(m, n, k, kp, g, packed)) return invalid("pair GEMV (config 13) does not take this shape");
    const int64_t xstride = cdiv(kp, 128) * 128 + gemv_xpad(g);
    const size_t xbytes = (size_t)(m * xstride) * sizeof(XT);
    const bool xs = (int64_t)xbytes <= kTileXs;
    const size_t sbytes = (size_t)cdiv(16 * (L::kStageCols / g) * 4, 128) * 128;
    const size_t pitch = (L::kStageBytes + sbytes + 1023) / 1024 * 1024;
    const size_t cbytes = (SA && xs) ? (size_t)cdiv(kp, 128) * 16 * 4 : 0;  // bias table
    const size_t smem = 1024 + 2 * pitch + 16 + gemv_red_bytes(8, NT) + (xs ? xbytes : 0) + cbytes;
    const int64_t tiles = cdiv(n, 16);
    const int64_t grid = std::min<int64_t>(tiles, sm_count());
    CUtensorMap wmap, smap;
    bool stma = false;
    int rc = make_gemv_maps<8, 4>(packed, scales, n, kp, g, &wmap, &smap, &stma);
    if (rc != OQ_OK) return rc;
    if (half_scales) {
        // fp16 scales by TMA too: a box of the stage's groups x 16 rows
        // (2-byte elements, rows of groups * 2 bytes), read unswizzled
        const int64_t groups = kp / g, spr = L::kStageCols / g;
        stma = (groups * 2) % 16 == 0 && (spr * 2) % 16 == 0 && aligned(scales, 16);
        if (stma) {
            rc = make_tensor_map_2d(&smap, scales, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)groups, (uint64_t)n,
                                    (uint64_t)(groups * 2), (uint32_t)spr, 16, CU_TENSOR_MAP_SWIZZLE_NONE);
            if (rc != OQ_OK) return rc;
        }
    }
    auto pick = [&](auto kern) -> int {
        int rc2 = allow_dynamic_smem(reinterpret_cast<const void *>(kern), smem);
        if (rc2 != OQ_OK) return rc2;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)grid);
        cfg.blockDim = dim3(512);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        cudaError_t err = cudaLaunchKernelEx(&cfg, kern, wmap, smap, x, scales, y, (int)m, (int)n, (int)k, (int)kp,
                                             gshift, (int)xstride, prefetch, half_scales ? 1 : 0);
        if (err != cudaSuccess) {
            set_error("int4_linear (pair GEMV): launch failed: %s", cudaGetErrorString(err));
            return OQ_ERR_CUDA;
        }
        return OQ_OK;
    };
    if (xs)
        return stma ? pick(gemv_pair_kernel<XT, NT, SA, true, true>) : pick(gemv_pair_kernel<XT, NT, SA, true, false>);
    return stma ? pick(gemv_pair_kernel<XT, NT, SA, false, true>) : pick(gemv_pair_kernel<XT, NT, SA, false, false>);
}

// True when the TMA GEMV takes this shape (M <= 16, 32 <= g <= the stage
// width, packed rows 16-byte aligned, and the shared-memory plan fits).
template <int CW, int CPW, int CTAS = 1>
bool tma_gemv_ok(int64_t m, int64_t k, int64_t kp, int g, const uint8_t *packed) {
    size_t smem = 0;
    int xstride = 0;
    bool xs = false;
    int nred = 2;
    return m <= 16 && aligned(packed, 16) && (kp / 2) % 16 == 0 &&
           tma_gemv_plan<CW, CPW>(m, k, kp, g, (int)((m + 7) / 8), 2, &smem, &xstride, &xs, &nred, CTAS) > 0;
}

// GEMV launch shapes, selected by the low bits of oq_int4_linear's
// `config` (0 = automatic):
//   1..7  register-ring kernel, (warps per CTA, chunks in flight per warp,
//         CTAs per SM) = (8,4,2) (16,2,2) (12,2,2) (16,1,2) (8,2,3) (8,2,4)
//         (8,4,4)
//   8, 9  TMA-fed persistent kernel with 8 / 16 consumer warps, 32 KB
//         stages (M <= 16)
//   10    TMA-fed, 8 consumer warps, two CTAs per SM with the stage ring
//         sized to the CTA's work
//   12    one CTA of 8 warps per 16-row tile, no producer warp, four CTAs
//         per SM (KP <= 4096, M <= 16): the next launch's CTAs fit beside
//         this one's, so back-to-back GEMVs overlap (PDL)
//   13    one CTA of 16 warps per SM owning two tiles (KP <= 4096, at most
//         two tiles per SM, M <= 16): balanced placement in back-to-back
//         launches, the next launch's weights stream meanwhile
// config & 16 (OQ_CONFIG_EXACT_ROUNDING) forces the exact weight rounding
// for fp16 x, which otherwise uses the scale-after path when g % 128 == 0.
// config & 32 (OQ_CONFIG_STATIC_WEIGHTS) lets the weights and scales stream
// before the wait on the previous kernel in the stream.
constexpr int kGemvConfigs = 13;

template <typename XT, int NT, bool SA>
int launch_gemv_nt(int config, const XT *x, const uint8_t *packed, const float *scales, OutSpec y, int64_t m,
                   int64_t n, int64_t k, int64_t kp, int g, int gshift, int pf, cudaStream_t st) {
    switch (config) {
        case 1: return launch_gemv_t<XT, NT, 8, 4, 2, SA>(x, packed, scales, y, m, n, k, kp, gshift, pf, st);
        case 2: return launch_gemv_t<XT, NT, 16, 2, 2, SA>(x, packed, scales, y, m, n, k, kp, gshift, pf, st);
        case 3: return launch_gemv_t<XT, NT, 12, 2, 2, SA>(x, packed, scales, y, m, n, k, kp, gshift, pf, st);
        case 4: return launch_gemv_t<XT, NT, 16, 1, 2, SA>(x, packed, scales, y, m, n, k, kp, gshift, pf, st);
        case 6: return launch_gemv_t<XT, NT, 8, 2, 4, SA>(x, packed, scales, y, m, n, k, kp, gshift, pf, st);
        case 7: return launch_gemv_t<XT, NT, 8, 4, 4, SA>(x, packed, scales, y, m, n, k, kp, gshift, pf, st);
        case 8:
            if constexpr (NT <= 2) return launch_gemv_tma<XT, NT, 8, 4, SA>(x, packed, scales, y, m, n, k, kp, g, gshift, pf, st);
            return invalid("TMA GEMV needs M <= 16");
        case 9:
            if constexpr (NT <= 2) return launch_gemv_tma<XT, NT, 16, 2, SA>(x, packed, scales, y, m, n, k, kp, g, gshift, pf, st);
            return invalid("TMA GEMV needs M <= 16");
        case 10:
            if constexpr (NT <= 2)
                return launch_gemv_tma<XT, NT, 8, 4, SA, 2>(x, packed, scales, y, m, n, k, kp, g, gshift, pf, st);
            return invalid("TMA GEMV needs M <= 16");
        case 12:
            if constexpr (NT <= 2) return launch_gemv_tile<XT, NT, SA>(x, packed, scales, y, m, n, k, kp, g, gshift, pf, st);
            return invalid("tile GEMV needs M <= 16");
        case 13:
            if constexpr (NT <= 2) return launch_gemv_pair<XT, NT, SA>(x, packed, scales, y, m, n, k, kp, g, gshift, pf, st);
            return invalid("pair GEMV needs M <= 16");
        default: return launch_gemv_t<XT, NT, 8, 2, 3, SA>(x, packed, scales, y, m, n, k, kp, gshift, pf, st);
    }
}

template <typename XT, bool SA>
int launch_gemv_sa(int shape, const XT *x, const uint8_t *packed, const float *scales, OutSpec y, int64_t m,
                   int64_t n, int64_t k, int64_t kp, int g, int gshift, int pf, cudaStream_t st) {
    switch ((m + 7) / 8) {
        case 1: return launch_gemv_nt<XT, 1, SA>(shape, x, packed, scales, y, m, n, k, kp, g, gshift, pf, st);
        case 2: return launch_gemv_nt<XT, 2, SA>(shape, x, packed, scales, y, m, n, k, kp, g, gshift, pf, st);
        case 3: case 4: return launch_gemv_nt<XT, 4, SA>(shape, x, packed, scales, y, m, n, k, kp, g, gshift, pf, st);
        default: return launch_gemv_t<XT, 8, 8, 2, 1, SA>(x, packed, scales, y, m, n, k, kp, gshift, pf, st);
    }
}

template <typename XT>
int launch_gemv(const XT *x, const uint8_t *packed, const float *scales, OutSpec y, int64_t m, int64_t n, int64_t k,
                int64_t kp, int g, int config, cudaStream_t st) {
    int gshift = 0;
    while ((1 << gshift) < g) ++gshift;
    const int nt = (int)((m + 7) / 8);
    int shape = config & 15;
    const bool auto_shape = shape <= 0 || shape > kGemvConfigs;
    if (auto_shape) {
        if (gemv_pair_ok(m, n, k, kp, g, packed))
            shape = 13;
        else if (nt == 1 && kp <= TmaGemvLayout<8, 4>::kStageCols && tma_gemv_ok<8, 4, 2>(m, k, kp, g, packed))
            shape = 10;
        else if (tma_gemv_ok<16, 2>(m, k, kp, g, packed))
            shape = 9;
        else if (tma_gemv_ok<8, 4>(m, k, kp, g, packed))
            shape = 8;
        else
            shape = nt <= 2 ? 1 : 5;
    }
    if ((shape == 8 && !tma_gemv_ok<8, 4>(m, k, kp, g, packed)) || (shape == 9 && !tma_gemv_ok<16, 2>(m, k, kp, g, packed)) ||
        (shape == 10 && !tma_gemv_ok<8, 4, 2>(m, k, kp, g, packed)))
        return invalid("TMA GEMV (config %d) does not take this shape", shape);
    if (shape == 11) return invalid("GEMV config 11 is not a launch shape");
    // Scale-after is the fp16 default up to M = 16 (two n-tiles): with the
    // conflict-free ldsm_x4 loads it beats the exact rounding there too (45 MB
    // layer at M = 16: 26.3 vs 30.6 us).
    const bool exact = (config & OQ_CONFIG_EXACT_ROUNDING) != 0 || (auto_shape && nt > 2);
    const int pf = (config & OQ_CONFIG_STATIC_WEIGHTS) != 0;
    if constexpr (std::is_same<XT, __half>::value) {
        if (!exact && g % 128 == 0)
            return launch_gemv_sa<XT, true>(shape, x, packed, scales, y, m, n, k, kp, g, gshift, pf, st);
    }
    return launch_gemv_sa<XT, false>(shape, x, packed, scales, y, m, n, k, kp, g, gshift, pf, st);
}

// fp16-scale variant (oq_int4_linear_f16s): fp16 x, scale-after mode (g % 128
// == 0), M <= 16, on the pair GEMV when it takes the shape, else the TMA GEMV
// with 16 consumer warps (or 8); each lane loads its rows' fp16 scales.
int launch_gemv_f16s(const __half *x, const uint8_t *packed, const float *scales16, OutSpec y, int64_t m, int64_t n,
                     int64_t k, int64_t kp, int g, int config, cudaStream_t st) {
    int gshift = 0;
    while ((1 << gshift) < g) ++gshift;
    const int pf = (config & OQ_CONFIG_STATIC_WEIGHTS) != 0;
    const bool two = m > 8;
    if (gemv_pair_ok(m, n, k, kp, g, packed))
        return two ? launch_gemv_pair<__half, 2, true>(x, packed, scales16, y, m, n, k, kp, g, gshift, pf, st, true)
                   : launch_gemv_pair<__half, 1, true>(x, packed, scales16, y, m, n, k, kp, g, gshift, pf, st, true);
    if (tma_gemv_ok<16, 2>(m, k, kp, g, packed))
        return two ? launch_gemv_tma<__half, 2, 16, 2, true>(x, packed, scales16, y, m, n, k, kp, g, gshift, pf, st, 0, true)
                   : launch_gemv_tma<__half, 1, 16, 2, true>(x, packed, scales16, y, m, n, k, kp, g, gshift, pf, st, 0, true);
    if (tma_gemv_ok<8, 4>(m, k, kp, g, packed))
        return two ? launch_gemv_tma<__half, 2, 8, 4, true>(x, packed, scales16, y, m, n, k, kp, g, gshift, pf, st, 0, true)
                   : launch_gemv_tma<__half, 1, 8, 4, true>(x, packed, scales16, y, m, n, k, kp, g, gshift, pf, st, 0, true);
    return invalid("fp16 scales: neither the pair nor the TMA GEMV takes this shape (x must fit in shared memory)");
}

// SiLU-gate mode (OQ_CONFIG_SILU_GATE): the TMA GEMV over the [gate; up]
// stack of 2 * n_out rows, y = silu(x . Wg^T) * (x . Wu^T).  The launch
// shape is config's (8, 9 or 10) or, for 0, the first of 10 (M <= 8, KP <= 4096), 9, 8
// that takes the shape.
template <typename XT>
int launch_gemv_gate(const XT *x, const uint8_t *packed, const float *scales, OutSpec y, int64_t m, int64_t n_out,
                     int64_t k, int64_t kp, int g, int config, cudaStream_t st) {
    int gshift = 0;
    while ((1 << gshift) < g) ++gshift;
    const int nt = (int)((m + 7) / 8);
    if (nt > 2) return invalid("SiLU-gate GEMV needs M <= 16");
    int shape = config & 15;
    const bool auto_shape = shape == 0;
    if (auto_shape) {
        if (nt == 1 && kp <= TmaGemvLayout<8, 4>::kStageCols && tma_gemv_ok<8, 4, 2>(m, k, kp, g, packed))
            shape = 10;
        else if (tma_gemv_ok<16, 2>(m, k, kp, g, packed))
            shape = 9;
        else if (tma_gemv_ok<8, 4>(m, k, kp, g, packed))
            shape = 8;
    }
    const bool fits = (shape == 8 && tma_gemv_ok<8, 4>(m, k, kp, g, packed)) ||
                      (shape == 9 && tma_gemv_ok<16, 2>(m, k, kp, g, packed)) ||
                      (shape == 10 && tma_gemv_ok<8, 4, 2>(m, k, kp, g, packed));
    if (!fits) return invalid("SiLU-gate GEMV: the TMA GEMV (config 8, 9 or 10) does not take this shape");
    const bool exact = (config & OQ_CONFIG_EXACT_ROUNDING) != 0 || (auto_shape && nt > 2);
    const int pf = (config & OQ_CONFIG_STATIC_WEIGHTS) != 0;
    const int64_t n2 = 2 * n_out;
    auto go = [&](auto sa_tag) -> int {
        constexpr bool SA = decltype(sa_tag)::value;
        if (nt == 1) {
            if (shape == 8) return launch_gemv_tma<XT, 1, 8, 4, SA>(x, packed, scales, y, m, n2, k, kp, g, gshift, pf, st, n_out);
            if (shape == 9) return launch_gemv_tma<XT, 1, 16, 2, SA>(x, packed, scales, y, m, n2, k, kp, g, gshift, pf, st, n_out);
            return launch_gemv_tma<XT, 1, 8, 4, SA, 2>(x, packed, scales, y, m, n2, k, kp, g, gshift, pf, st, n_out);
        }
        if (shape == 8) return launch_gemv_tma<XT, 2, 8, 4, SA>(x, packed, scales, y, m, n2, k, kp, g, gshift, pf, st, n_out);
        if (shape == 9) return launch_gemv_tma<XT, 2, 16, 2, SA>(x, packed, scales, y, m, n2, k, kp, g, gshift, pf, st, n_out);
        return launch_gemv_tma<XT, 2, 8, 4, SA, 2>(x, packed, scales, y, m, n2, k, kp, g, gshift, pf, st, n_out);
    };
    if constexpr (std::is_same<XT, __half>::value) {
        if (!exact && g % 128 == 0) return go(std::true_type{});
    }
    return go(std::false_type{});
}

template <typename XT>
int launch_simt(const XT *x, const uint8_t *packed, const float *scales, OutSpec y, int64_t m, int64_t n, int64_t k,
                int64_t kp, int g, cudaStream_t st) {
    int64_t blocks = cdiv(n, 8);
    const int64_t cap = (int64_t)sm_count() * 8;
    if (blocks > cap) blocks = cap;
    simt_int4_kernel<XT><<<(unsigned)blocks, 256, 0, st>>>(x, packed, scales, y, m, n, k, kp, g);
    return check_launch("int4_linear (SIMT)");
}

}  // namespace

bool gemv_supported(int64_t m, int64_t n, int64_t k, int g, const void *x, const uint8_t *packed) {
    if (!(m >= 1 && m <= 64 && g >= 32 && (g & (g - 1)) == 0 && k % 8 == 0 && aligned(x, 16) &&
          aligned(packed, 16)))
        return false;
    const int64_t kp = cdiv(k, g) * g;
    if (n >= (1ll << 31) || kp >= (1ll << 30) || n * (kp / 2) >= (1ll << 40)) return false;
    // x from global memory needs KP == K and whole 128-column chunks.
    return gemv_xs_bytes(m, kp, 2) > 0 || (kp == k && kp % 128 == 0);
}

}  // namespace oq

using namespace oq;

namespace oq {
namespace {

// The kernel the automatic choice (and an explicit `kernel`) runs.
int choose_kernel(int64_t m, int64_t n, int64_t k, int group_size, const void *x, const uint8_t *packed,
                  int kernel) {
    if (kernel != OQ_KERNEL_AUTO) return kernel;
    const bool gemv_ok = gemv_supported(m, n, k, group_size, x, packed);
    if (gemv_ok && m <= 16) return OQ_KERNEL_GEMV;
    if (gemm_tcgen05_supported(m, n, k, group_size, x, packed, nullptr)) return OQ_KERNEL_TCGEN05;
    return gemv_ok ? OQ_KERNEL_GEMV : OQ_KERNEL_SIMT;
}

int int4_linear_impl(const void *x, int x_dtype, const uint8_t *packed, const float *scales, OutSpec y, int64_t m,
                     int64_t n, int64_t k, int group_size, int kernel, int config, void *ws, size_t ws_bytes,
                     oq_stream_t stream) {
    OQ_REQUIRE(x_dtype == OQ_F16 || x_dtype == OQ_BF16, "Input must be a 2D FP16 or BF16 tensor");
    OQ_REQUIRE(group_size >= 2 && group_size % 2 == 0, "Group size must be even and >= 2");
    OQ_REQUIRE(m >= 1 && n >= 1 && k >= 1, "Matrix dimensions must be positive");
    OQ_REQUIRE(x && packed && scales && y.y, "null pointer argument");
    OQ_REQUIRE(y.dtype == OQ_F32 || y.dtype == OQ_F16 || y.dtype == OQ_BF16, "output dtype must be fp32, fp16 or bf16");
    if (y.ld == 0) y.ld = n;
    OQ_REQUIRE(y.col0 >= 0 && y.col0 + n <= y.ld, "output columns [col0, col0 + n) must lie in a row of ld");
    const int64_t kp = cdiv(k, group_size) * group_size;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (config & OQ_CONFIG_SILU_GATE) {
        OQ_REQUIRE(kernel == OQ_KERNEL_AUTO || kernel == OQ_KERNEL_GEMV || kernel == OQ_KERNEL_TCGEN05,
                   "SiLU-gate fusion runs on the GEMV (M <= 16) or the tcgen05 GEMM");
        OQ_REQUIRE(y.bias == nullptr, "SiLU-gate fusion takes no bias");
        OQ_REQUIRE(n < (1ll << 30), "SiLU-gate fusion: too many features");
        const bool on_gemv = kernel == OQ_KERNEL_GEMV || (kernel == OQ_KERNEL_AUTO && m <= 16 &&
                                                          gemv_supported(m, 2 * n, k, group_size, x, packed));
        if (!on_gemv) {
            OQ_REQUIRE(gemm_tcgen05_supported(m, 2 * n, k, group_size, x, packed, nullptr),
                       "SiLU-gate fusion: the tcgen05 GEMM does not take this shape/alignment");
            return gemm_tcgen05_launch(x, x_dtype, packed, scales, y, m, 2 * n, k, group_size, nullptr, 0, st, n);
        }
        OQ_REQUIRE(m <= 16 && gemv_supported(m, 2 * n, k, group_size, x, packed),
                   "SiLU-gate fusion on the GEMV needs M <= 16 and a shape the GEMV takes");
        if (x_dtype == OQ_F16)
            return launch_gemv_gate(static_cast<const __half *>(x), packed, scales, y, m, n, k, kp, group_size, config, st);
        return launch_gemv_gate(static_cast<const __nv_bfloat16 *>(x), packed, scales, y, m, n, k, kp, group_size,
                                config, st);
    }
    const bool gemv_ok = gemv_supported(m, n, k, group_size, x, packed);
    const int which = choose_kernel(m, n, k, group_size, x, packed, kernel);
    switch (which) {
        case OQ_KERNEL_GEMV:
            OQ_REQUIRE(gemv_ok, "GEMV kernel needs M <= 64, a power-of-two group_size >= 32, K % 8 == 0, 16-byte aligned x/packed, and x staged in shared memory or K a multiple of 128 and of the group");
            if (x_dtype == OQ_F16)
                return launch_gemv(static_cast<const __half *>(x), packed, scales, y, m, n, k, kp, group_size, config,
                                   st);
            return launch_gemv(static_cast<const __nv_bfloat16 *>(x), packed, scales, y, m, n, k, kp, group_size,
                               config, st);
        case OQ_KERNEL_TCGEN05:
            OQ_REQUIRE(gemm_tcgen05_supported(m, n, k, group_size, x, packed, nullptr),
                       "tcgen05 kernel does not support this shape/alignment");
            return gemm_tcgen05_launch(x, x_dtype, packed, scales, y, m, n, k, group_size, ws, ws_bytes, st);
        case OQ_KERNEL_SIMT:
            if (x_dtype == OQ_F16)
                return launch_simt(static_cast<const __half *>(x), packed, scales, y, m, n, k, kp, group_size, st);
            return launch_simt(static_cast<const __nv_bfloat16 *>(x), packed, scales, y, m, n, k, kp, group_size, st);
        default:
            return invalid("unknown kernel selector %d", kernel);
    }
}

}  // namespace
}  // namespace oq

extern "C" int oq_int4_linear(const void *x, int x_dtype, const uint8_t *packed, const float *scales, float *y,
                              int64_t m, int64_t n, int64_t k, int group_size, int kernel, int config,
                              oq_stream_t stream) {
    clear_error();
    return int4_linear_impl(x, x_dtype, packed, scales, OutSpec{y, nullptr, OQ_F32}, m, n, k, group_size, kernel,
                            config, nullptr, 0, stream);
}

extern "C" int oq_int4_linear_ex(const void *x, int x_dtype, const uint8_t *packed, const float *scales, void *y,
                                 int y_dtype, const float *bias, int64_t m, int64_t n, int64_t k, int group_size,
                                 int kernel, int config, oq_stream_t stream) {
    clear_error();
    return int4_linear_impl(x, x_dtype, packed, scales, OutSpec{y, bias, y_dtype}, m, n, k, group_size, kernel,
                            config, nullptr, 0, stream);
}

extern "C" int oq_int4_linear_ws(const void *x, int x_dtype, const uint8_t *packed, const float *scales, void *y,
                                 int y_dtype, const float *bias, int64_t m, int64_t n, int64_t k, int group_size,
                                 int kernel, int config, void *workspace, size_t ws_bytes, oq_stream_t stream) {
    clear_error();
    OQ_REQUIRE(workspace == nullptr || aligned(workspace, 16), "workspace must be 16-byte aligned");
    return int4_linear_impl(x, x_dtype, packed, scales, OutSpec{y, bias, y_dtype}, m, n, k, group_size, kernel,
                            config, workspace, ws_bytes, stream);
}

extern "C" int oq_int4_linear_f16s(const void *x, int x_dtype, const uint8_t *packed, const void *scales, void *y,
                                   int y_dtype, const float *bias, int64_t m, int64_t n, int64_t k, int group_size,
                                   int config, oq_stream_t stream) {
    clear_error();
    OQ_REQUIRE(x_dtype == OQ_F16, "fp16 scales take fp16 x");
    OQ_REQUIRE(group_size >= 2 && group_size % 2 == 0, "Group size must be even and >= 2");
    OQ_REQUIRE(m >= 1 && n >= 1 && k >= 1, "Matrix dimensions must be positive");
    OQ_REQUIRE(x && packed && scales && y, "null pointer argument");
    OQ_REQUIRE(y_dtype == OQ_F32 || y_dtype == OQ_F16 || y_dtype == OQ_BF16, "output dtype must be fp32, fp16 or bf16");
    OQ_REQUIRE(aligned(scales, 2), "fp16 scales must be 2-byte aligned");
    OQ_REQUIRE(m <= 16 && group_size % 128 == 0 && gemv_supported(m, n, k, group_size, x, packed),
               "fp16 scales run on the decode GEMV: M <= 16, a power-of-two group size that is a multiple of 128, "
               "K %% 8 == 0, 16-byte aligned x and packed");
    OutSpec out{y, bias, y_dtype};
    out.ld = n;
    const int64_t kp = cdiv(k, group_size) * group_size;
    return launch_gemv_f16s(static_cast<const __half *>(x), packed, static_cast<const float *>(scales), out, m, n, k,
                            kp, group_size, config, static_cast<cudaStream_t>(stream));
}

namespace oq {
namespace {
// Device address of page-locked host memory (the same pointer on a
// unified-address system), or nullptr when `p` is not page-locked and mapped.
void *mapped_host_address(const void *p) {
    cudaPointerAttributes attr{};
    if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
        cudaGetLastError();  // pageable memory: not an error state to keep
        return nullptr;
    }
    if (attr.type != cudaMemoryTypeHost || attr.devicePointer == nullptr) return nullptr;
    return attr.devicePointer;
}

// Copies `bytes` from mapped host memory into device memory (both addresses
// 16-byte aligned), 16 bytes per thread and the last bytes % 16 by thread 0:
// one read of the activations over the bus per decode step, after which
// every CTA of the layer kernel reads them from L2.  It lets the layer kernel
// launch at once (programmatic dependent launch), so the kernel's static
// weights stream from HBM while the activations cross the bus.
__global__ void __launch_bounds__(256) host_to_device_kernel(const uint8_t *__restrict__ src,
                                                              uint8_t *__restrict__ dst, int64_t bytes) {
    asm volatile("griddepcontrol.launch_dependents;");
    const int64_t n16 = bytes / 16;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n16) reinterpret_cast<uint4 *>(dst)[i] = reinterpret_cast<const uint4 *>(src)[i];
    if (i == 0)
        for (int64_t b = n16 * 16; b < bytes; ++b) dst[b] = src[b];
}
}  // namespace
}  // namespace oq

namespace oq {
namespace {
// Validates a host-buffer call and enqueues it on `st`: the copy kernel,
// then the layer kernel writing y through its mapped address.
int host_enqueue(const void *x, int x_dtype, const uint8_t *packed, const float *scales, void *y, int y_dtype,
                 const float *bias, int64_t m, int64_t n, int64_t k, int group_size, int kernel, int config,
                 void *x_stage, cudaStream_t st) {
    OQ_REQUIRE(x && y && packed && scales && x_stage, "null pointer argument");
    void *xd = mapped_host_address(x);
    void *yd = mapped_host_address(y);
    OQ_REQUIRE(xd != nullptr && yd != nullptr,
               "x and y must be page-locked host memory (cudaHostAlloc / cudaHostRegister; torch: pin_memory())");
    OQ_REQUIRE(x_dtype == OQ_F16 || x_dtype == OQ_BF16, "Input must be a 2D FP16 or BF16 tensor");
    OQ_REQUIRE(m >= 1 && n >= 1 && k >= 1 && m < (1ll << 40) / k, "Matrix dimensions must be positive");
    const int64_t xbytes = m * k * 2;
    OQ_REQUIRE(aligned(xd, 16) && aligned(x_stage, 16), "host input: x and x_stage must be 16-byte aligned");
    host_to_device_kernel<<<(unsigned)std::max<int64_t>(1, cdiv(xbytes / 16, 256)), 256, 0, st>>>(
        static_cast<const uint8_t *>(xd), static_cast<uint8_t *>(x_stage), xbytes);
    const int rc = check_launch("int4_linear (host input copy)");
    if (rc != OQ_OK) return rc;
    return int4_linear_impl(x_stage, x_dtype, packed, scales, OutSpec{yd, bias, y_dtype}, m, n, k, group_size, kernel,
                            config, nullptr, 0, st);
}

// A captured host-buffer call (oq_int4_linear_host_plan).
struct HostPlan {
    cudaGraphExec_t exec = nullptr;
    int device = -1;
};
}  // namespace
}  // namespace oq

extern "C" int oq_int4_linear_host_plan(const void *x, int x_dtype, const uint8_t *packed, const float *scales,
                                        void *y, int y_dtype, const float *bias, int64_t m, int64_t n, int64_t k,
                                        int group_size, int kernel, int config, void *x_stage, void **plan) {
    clear_error();
    OQ_REQUIRE(plan != nullptr, "null plan pointer");
    *plan = nullptr;
    int dev = 0;
    OQ_CUDA(cudaGetDevice(&dev));
    cudaStream_t cs = nullptr;
    OQ_CUDA(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking));
    cudaGraph_t graph = nullptr;
    cudaError_t err = cudaStreamBeginCapture(cs, cudaStreamCaptureModeRelaxed);
    int rc = OQ_OK;
    if (err == cudaSuccess) {
        rc = host_enqueue(x, x_dtype, packed, scales, y, y_dtype, bias, m, n, k, group_size, kernel, config, x_stage,
                          cs);
        const cudaError_t end = cudaStreamEndCapture(cs, &graph);  // ends the capture whatever happened
        if (rc == OQ_OK && end != cudaSuccess) err = end;
    }
    cudaGraphExec_t exec = nullptr;
    if (err == cudaSuccess && rc == OQ_OK) err = cudaGraphInstantiate(&exec, graph, 0);
    if (graph) cudaGraphDestroy(graph);
    cudaStreamDestroy(cs);
    if (rc != OQ_OK) return rc;
    if (err != cudaSuccess) {
        set_error("int4_linear host plan: graph capture failed: %s", cudaGetErrorString(err));
        return OQ_ERR_CUDA;
    }
    auto *hp = new HostPlan;
    hp->exec = exec;
    hp->device = dev;
    *plan = hp;
    return OQ_OK;
}

extern "C" int oq_int4_linear_host_run(void *plan, oq_stream_t stream) {
    clear_error();
    OQ_REQUIRE(plan != nullptr, "null plan");
    auto *hp = static_cast<HostPlan *>(plan);
    int dev = 0;
    OQ_CUDA(cudaGetDevice(&dev));
    OQ_REQUIRE(dev == hp->device, "the plan was made on device %d, the current device is %d", hp->device, dev);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    OQ_CUDA(cudaGraphLaunch(hp->exec, st));
    OQ_CUDA(cudaStreamSynchronize(st));
    return OQ_OK;
}

extern "C" int oq_int4_linear_host_plan_free(void *plan) {
    clear_error();
    if (plan == nullptr) return OQ_OK;
    auto *hp = static_cast<HostPlan *>(plan);
    const cudaError_t err = cudaGraphExecDestroy(hp->exec);
    delete hp;
    OQ_CUDA(err);
    return OQ_OK;
}

extern "C" int oq_int4_linear_host(const void *x, int x_dtype, const uint8_t *packed, const float *scales, void *y,
                                   int y_dtype, const float *bias, int64_t m, int64_t n, int64_t k, int group_size,
                                   int kernel, int config, void *x_stage, oq_stream_t stream) {
    clear_error();
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int rc = host_enqueue(x, x_dtype, packed, scales, y, y_dtype, bias, m, n, k, group_size, kernel, config,
                                x_stage, st);
    if (rc != OQ_OK) return rc;
    OQ_CUDA(cudaStreamSynchronize(st));
    return OQ_OK;
}

extern "C" int64_t oq_int4_linear_workspace_bytes(int64_t m, int64_t n, int64_t k, int group_size, int kernel,
                                                  int config) {
    clear_error();
    if (m < 1 || n < 1 || k < 1 || group_size < 2 || (config & OQ_CONFIG_SILU_GATE)) return 0;
    // The GEMV and CUDA-core kernels take no workspace; the shapes the GEMM
    // takes are alignment-independent apart from x / packed (16 bytes).
    static const uint8_t aligned_probe[16] __attribute__((aligned(16))) = {};
    const int which = choose_kernel(m, n, k, group_size, aligned_probe, aligned_probe, kernel);
    if (which != OQ_KERNEL_TCGEN05 || !gemm_tcgen05_supported(m, n, k, group_size, aligned_probe, aligned_probe, nullptr))
        return 0;
    return (int64_t)gemm_tcgen05_workspace_bytes(m, n, k, group_size);
}

extern "C" int oq_int4_linear_peers(const void *x, int x_dtype, const uint8_t *packed, const float *scales,
                                    void *const *y_gpus, int n_gpus, int y_dtype, const float *bias, int64_t ld,
                                    int64_t col0, int64_t m, int64_t n, int64_t k, int group_size, int kernel,
                                    int config, void *workspace, size_t ws_bytes, oq_stream_t stream) {
    clear_error();
    OQ_REQUIRE(y_gpus != nullptr && n_gpus >= 1 && n_gpus <= kMaxOutGpus, "n_gpus must be in [1, %d]", kMaxOutGpus);
    OQ_REQUIRE(ld >= 1 && col0 >= 0 && col0 + n <= ld, "output columns [col0, col0 + n) must lie in a row of ld");
    OQ_REQUIRE(m < (1ll << 40) / ld, "output too large");
    OutSpec out{y_gpus[0], bias, y_dtype};
    out.npeers = n_gpus - 1;
    out.ld = ld;
    out.col0 = col0;
    for (int i = 1; i < n_gpus; ++i) {
        OQ_REQUIRE(y_gpus[i] != nullptr, "null output pointer for GPU %d", i);
        out.peer[i - 1] = y_gpus[i];
    }
    OQ_REQUIRE(workspace == nullptr || aligned(workspace, 16), "workspace must be 16-byte aligned");
    return int4_linear_impl(x, x_dtype, packed, scales, out, m, n, k, group_size, kernel, config, workspace, ws_bytes,
                            stream);
}
