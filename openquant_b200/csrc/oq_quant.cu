// Quantize and dequantize kernels: per-row INT8, per-row flat-packed INT4 and
// groupwise INT4 (openquant 0.5.0 formats), sm_100a.
//
// All of these are HBM-streaming kernels: 16-byte vector loads of 8
// consecutive weights per thread, warp-shuffle max reductions, 4-/8-byte
// packed stores.  Bit-exactness with the reference rests on oq::quant_bits()
// (IEEE quotient, round-half-even) and oq::scale_from_max() (IEEE division).
#include "oq_sm100.cuh"

#include <algorithm>
#include <type_traits>

namespace oq {
namespace {

constexpr int kRowThreads = 256;

// ------------------------------------------------------------ helpers --

template <typename T> __device__ __forceinline__ float ld(const T *p, int64_t i) {
    return Elem<T>::to_f32(p[i]);
}

// Block-wide NaN-propagating max; every thread gets the result.
__device__ __forceinline__ float block_max(float v, float *smem) {
    v = warp_max(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) smem[warp] = v;
    __syncthreads();
    const int nw = blockDim.x >> 5;
    float r = lane < nw ? smem[lane] : 0.0f;
    r = warp_max(r);
    __syncthreads();
    return r;
}

// Near-tie bound of the reciprocal fast paths.  With a normal scale s and
// |v| <= max, r = fl(v * fl(1/s)) and the reference quotient fl(v / s) each
// lie within 7 * 2^-23 of v/s, so |r - fl(v/s)| < 2^-19.  Their roundings
// can only differ if a half-integer lies between them, i.e. if r is within
// 2^-19 of a tie; |d| = |r - rint(r)| >= 0.5 - 2^-16 covers that 8x over.
// The bound is tight so that a warp-wide vote rarely takes the exact path.
constexpr float kNearTie = 0.5f - 1.0f / 65536.0f;
constexpr float kNearTieSq = kNearTie * kNearTie;

// Eight quotients q_i = clip(rint(fl(v_i / s)), -qmax, qmax) as the bit
// patterns of (q_i + 1.5*2^23) (low byte / nibble = q_i), like quant_bits but
// with packed f32x2 arithmetic: r = v * (1/s), t = r + 1.5*2^23 (round half
// to even), d = r - (t - 1.5*2^23).  When any lane of `mask` has a quotient
// near a tie (|d| >= kNearTie) or a scale that is not a normal float
// (zero-substituted, subnormal, NaN), those lanes redo all eight with
// quant_bits (IEEE quotient, clipping, NaN -> 0).  For a normal scale derived
// from the values' max, |v/s| <= qmax up to a few ulps, so no clip is needed.
__device__ __forceinline__ void quant8(const float (&v)[8], float s, float inv, float qmax, uint32_t (&bits)[8],
                                       unsigned mask) {
    const float2 magic2 = make_float2(kRoundMagic, kRoundMagic);
    const float2 nmagic2 = make_float2(-kRoundMagic, -kRoundMagic);
    const float2 inv2 = make_float2(inv, inv);
    bool slow = !(s >= 1.17549435e-38f);
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const float2 rq = __fmul2_rn(make_float2(v[2 * p], v[2 * p + 1]), inv2);
        const float2 tt = __fadd2_rn(rq, magic2);
        const float2 rr = __fadd2_rn(tt, nmagic2);
        const float2 d = __ffma2_rn(rr, make_float2(-1.0f, -1.0f), rq);  // rq - rr, exact
        slow |= !(fabsf(d.x) < kNearTie) | !(fabsf(d.y) < kNearTie);
        bits[2 * p] = __float_as_uint(tt.x);
        bits[2 * p + 1] = __float_as_uint(tt.y);
    }
    if (__any_sync(mask, slow)) {
#pragma unroll
        for (int i = 0; i < 8; ++i) bits[i] = quant_bits(v[i], s, inv, qmax);
    }
}

// ---------------------------------------------- per-row quantize kernels --

// One CTA per row.  Pass 1 reduces max|w| over the row, pass 2 re-reads the
// row (an L2 hit: the resident rows are a few tens of MB) and quantizes.
// BITS = 8 writes int8; BITS = 4 writes the row's bytes of the flat packing
// that lie entirely inside the row (quantization.py:41-52).  With odd K the
// bytes that straddle two rows are written by straddle_kernel afterwards.
template <typename T, int BITS, bool VEC>
__global__ void __launch_bounds__(kRowThreads) quant_rowwise_kernel(const T *__restrict__ w, int64_t n,
                                                                    int64_t k, uint8_t *__restrict__ out,
                                                                    float *__restrict__ scales) {
    __shared__ float red[32];
    const float qmax = BITS == 8 ? 127.0f : 7.0f;
    const int64_t r = blockIdx.x;
    const T *row = w + r * k;

    float mx = 0.0f;
    if (VEC) {
        for (int64_t c = 8 * (int64_t)threadIdx.x; c < k; c += 8 * (int64_t)blockDim.x) {
            float v[8];
            load8<T>(row + c, v);
#pragma unroll
            for (int i = 0; i < 8; ++i) mx = nan_max(mx, fabsf(v[i]));
        }
    } else {
        for (int64_t c = threadIdx.x; c < k; c += blockDim.x) mx = nan_max(mx, fabsf(ld(row, c)));
    }
    mx = block_max(mx, red);
    const float s = scale_from_max(mx, qmax);
    const float inv = __frcp_rn(s);
    if (threadIdx.x == 0) scales[r] = s;

    if (BITS == 8) {
        int8_t *qrow = reinterpret_cast<int8_t *>(out) + r * k;
        if (VEC) {
            for (int64_t c = 8 * (int64_t)threadIdx.x; c < k; c += 8 * (int64_t)blockDim.x) {
                float v[8];
                load8<T>(row + c, v);
                uint32_t b[8];
                quant8(v, s, inv, qmax, b, __activemask());
                uint32_t lo = 0, hi = 0;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    lo |= (b[i] & 0xFFu) << (8 * i);
                    hi |= (b[i + 4] & 0xFFu) << (8 * i);
                }
                *reinterpret_cast<uint2 *>(qrow + c) = make_uint2(lo, hi);
            }
        } else {
            for (int64_t c = threadIdx.x; c < k; c += blockDim.x)
                qrow[c] = (int8_t)(quant_bits(ld(row, c), s, inv, qmax) & 0xFFu);
        }
    } else {
        if (VEC) {  // K % 8 == 0: the row owns bytes [r*K/2, r*K/2 + K/2)
            uint8_t *prow = out + r * (k / 2);
            for (int64_t c = 8 * (int64_t)threadIdx.x; c < k; c += 8 * (int64_t)blockDim.x) {
                float v[8];
                load8<T>(row + c, v);
                uint32_t b[8];
                quant8(v, s, inv, qmax, b, __activemask());
                uint32_t word = 0;
#pragma unroll
                for (int i = 0; i < 8; ++i) word |= (b[i] & 15u) << (4 * i);
                *reinterpret_cast<uint32_t *>(prow + c / 2) = word;
            }
        } else {
            // Bytes b with both elements 2b, 2b+1 inside row r.
            const int64_t f0 = r * k;
            const int64_t b0 = (f0 + 1) / 2, be = (f0 + k) / 2;
            for (int64_t b = b0 + threadIdx.x; b < be; b += blockDim.x) {
                const int64_t c = 2 * b - f0;
                uint32_t lo = quant_bits(ld(row, c), s, inv, qmax) & 15u;
                uint32_t hi = quant_bits(ld(row, c + 1), s, inv, qmax) & 15u;
                out[b] = (uint8_t)(lo | (hi << 4));
            }
            // Odd total: the last element is padded with a zero nibble.
            if (r == n - 1 && ((n * k) & 1) && threadIdx.x == 0) {
                out[(n * k - 1) / 2] = (uint8_t)(quant_bits(ld(row, k - 1), s, inv, qmax) & 15u);
            }
        }
    }
}

// Odd K: the byte holding (row r-1, col K-1) and (row r, col 0), for every
// row r >= 1 whose first flat index r*K is odd.
template <typename T>
__global__ void straddle_kernel(const T *__restrict__ w, int64_t n, int64_t k, uint8_t *__restrict__ out,
                                const float *__restrict__ scales) {
    for (int64_t r = 1 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r < n;
         r += (int64_t)gridDim.x * blockDim.x) {
        const int64_t f = r * k;
        if (!(f & 1)) continue;
        const float s0 = scales[r - 1], s1 = scales[r];
        uint32_t lo = quant_bits(ld(w, f - 1), s0, __frcp_rn(s0), 7.0f) & 15u;
        uint32_t hi = quant_bits(ld(w, f), s1, __frcp_rn(s1), 7.0f) & 15u;
        out[(f - 1) / 2] = (uint8_t)(lo | (hi << 4));
    }
}

// ------------------------------------------------ groupwise quantize --

// One thread per 8 padded columns; L = g/8 consecutive lanes form a group
// and reduce its max with shuffles (g in {8,16,...,256}).  Each thread
// writes one 32-bit word of the packed row (KP % 8 == 0 keeps it aligned).
template <typename T, int L, bool VEC>
__global__ void __launch_bounds__(256) quant_group_kernel(const T *__restrict__ w, int64_t n, int64_t k,
                                                          int64_t kp, uint8_t *__restrict__ packed,
                                                          float *__restrict__ scales,
                                                          int32_t *__restrict__ nonfinite) {
    const int64_t chunks_per_row = kp / 8;
    const int64_t total = n * chunks_per_row;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;  // a multiple of 32 and of L
    bool bad = false;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t - threadIdx.x % 32 < total;
         t += stride) {
        const bool live = t < total;
        const int64_t r = live ? t / chunks_per_row : 0;
        const int64_t j = live ? t - r * chunks_per_row : 0;
        const int64_t c0 = 8 * j;
        float v[8];
        if (live && VEC && c0 < k) {
            load8<T>(w + r * k + c0, v);
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = (live && c0 + i < k) ? ld(w, r * k + c0 + i) : 0.0f;
        }
        float mx = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            bad |= !isfinite(v[i]);
            mx = fmaxf(mx, fabsf(v[i]));
        }
#pragma unroll
        for (int o = L / 2; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const float s = scale_from_max(mx, 7.0f);
        const float inv = __frcp_rn(s);
        if (live) {
            if ((j % L) == 0) scales[r * (chunks_per_row / L) + j / L] = s;
            uint32_t word = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) word |= (quant_bits(v[i], s, inv, 7.0f) & 15u) << (4 * i);
            *reinterpret_cast<uint32_t *>(packed + r * (kp / 2) + 4 * j) = word;
        }
    }
    if (nonfinite != nullptr && bad) *nonfinite = 1;
}

// Fast groupwise quantizer (16-byte-aligned rows, K % 8 == 0): same
// thread/group mapping as quant_group_kernel, two 8-weight chunks in flight
// per thread, one fmax per weight for the group max, non-finite detection by
// a running fma(w, 0, acc) (NaN iff some w is NaN or +-Inf), and the packed
// f32x2 quotients of quant8().  Bit-exact with quant_group_kernel (and the
// reference) by construction.
template <typename T, int L>
__global__ void __launch_bounds__(256) quant_group_fast_kernel(const T *__restrict__ w, int64_t n, int64_t k,
                                                               int64_t kp, uint8_t *__restrict__ packed,
                                                               float *__restrict__ scales,
                                                               int32_t *__restrict__ nonfinite) {
    constexpr int C = 2;  // chunks per thread per iteration
    const int64_t chunks_per_row = kp / 8;
    const int64_t total = n * chunks_per_row;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;  // a multiple of 32 and of L
    float fin = 0.0f;
    for (int64_t t0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t0 - threadIdx.x % 32 < total;
         t0 += C * stride) {
        float v[C][8];
        int64_t r[C], j[C];
        bool live[C];
#pragma unroll
        for (int c = 0; c < C; ++c) {
            const int64_t t = t0 + c * stride;
            live[c] = t < total;
            r[c] = live[c] ? t / chunks_per_row : 0;
            j[c] = live[c] ? t - r[c] * chunks_per_row : 0;
            if (live[c] && 8 * j[c] < k) {
                load8<T>(w + r[c] * k + 8 * j[c], v[c]);
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) v[c][i] = 0.0f;
            }
        }
#pragma unroll
        for (int c = 0; c < C; ++c) {
            float mx = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                mx = fmaxf(mx, fabsf(v[c][i]));
                fin = fmaf(v[c][i], 0.0f, fin);
            }
#pragma unroll
            for (int o = L / 2; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            const float s = scale_from_max(mx, 7.0f);
            const float inv = __frcp_rn(s);
            uint32_t b[8];
            quant8(v[c], s, inv, 7.0f, b, 0xffffffffu);
            uint32_t word = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) word |= (b[i] & 15u) << (4 * i);
            if (live[c]) {
                if ((j[c] % L) == 0) scales[r[c] * (chunks_per_row / L) + j[c] / L] = s;
                *reinterpret_cast<uint32_t *>(packed + r[c] * (kp / 2) + 4 * j[c]) = word;
            }
        }
    }
    if (nonfinite != nullptr && fin != fin) *nonfinite = 1;
}

// ------------------------------------------- streaming groupwise quantize --
//
// For K % g == 0 (no padding) the weights, the packed nibbles and the scales
// are three flat arrays: weight e goes to byte e/2 and scale e/g.  The
// stream kernel walks the weights in 16 KB tiles: one producer lane keeps a
// ring of tiles in flight with 1-D bulk copies into shared memory (mbarrier
// completion, bounded waits), and CW consumer warps quantize each tile with
// every thread owning CPT consecutive 8-weight chunks of one group.

constexpr int kStreamTile = 16384;  // bytes per stage

// Raw 8-weight chunks: the integer |w| max (|w| bit patterns of IEEE types
// order like their values, Inf and NaN above every finite value) and the
// conversion of the raw words to f32.
template <typename T> struct Chunk;
template <> struct Chunk<__nv_bfloat16> {
    static constexpr int kWords = 4;
    static constexpr bool kCorrected = true;  // quot8's corrected quotient is exact for 16-bit weights
    static constexpr uint32_t kNonFinite = 0x7F80u;
    static __device__ __forceinline__ uint32_t absmax(const uint32_t *x) {
        return __vmaxu2(__vmaxu2(x[0] & 0x7FFF7FFFu, x[1] & 0x7FFF7FFFu),
                        __vmaxu2(x[2] & 0x7FFF7FFFu, x[3] & 0x7FFF7FFFu));
    }
    static __device__ __forceinline__ uint32_t combine(uint32_t a, uint32_t b) { return __vmaxu2(a, b); }
    static __device__ __forceinline__ uint32_t fold(uint32_t m) { return max(m & 0xFFFFu, m >> 16); }
    static __device__ __forceinline__ float to_f32(uint32_t m) { return __uint_as_float(m << 16); }
    static __device__ __forceinline__ void unpack(const uint32_t *x, float (&v)[8]) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            v[2 * i] = __uint_as_float(x[i] << 16);
            v[2 * i + 1] = __uint_as_float(x[i] & 0xFFFF0000u);
        }
    }
};
template <> struct Chunk<__half> {
    static constexpr int kWords = 4;
    static constexpr bool kCorrected = true;
    static constexpr uint32_t kNonFinite = 0x7C00u;
    static __device__ __forceinline__ uint32_t absmax(const uint32_t *x) { return Chunk<__nv_bfloat16>::absmax(x); }
    static __device__ __forceinline__ uint32_t combine(uint32_t a, uint32_t b) { return __vmaxu2(a, b); }
    static __device__ __forceinline__ uint32_t fold(uint32_t m) { return max(m & 0xFFFFu, m >> 16); }
    static __device__ __forceinline__ float to_f32(uint32_t m) { return __half2float(__ushort_as_half((unsigned short)m)); }
    static __device__ __forceinline__ void unpack(const uint32_t *x, float (&v)[8]) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            __half2 h;
            memcpy(&h, &x[i], 4);
            const float2 f = __half22float2(h);
            v[2 * i] = f.x;
            v[2 * i + 1] = f.y;
        }
    }
};
template <> struct Chunk<float> {
    static constexpr int kWords = 8;
    static constexpr bool kCorrected = false;
    static constexpr uint32_t kNonFinite = 0x7F800000u;
    static __device__ __forceinline__ uint32_t absmax(const uint32_t *x) {
        uint32_t m = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) m = max(m, x[i] & 0x7FFFFFFFu);
        return m;
    }
    static __device__ __forceinline__ uint32_t combine(uint32_t a, uint32_t b) { return max(a, b); }
    static __device__ __forceinline__ uint32_t fold(uint32_t m) { return m; }
    static __device__ __forceinline__ float to_f32(uint32_t m) { return __uint_as_float(m); }
    static __device__ __forceinline__ void unpack(const uint32_t *x, float (&v)[8]) {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(x[i]);
    }
};

// Rounded quotients of eight weights, rr_i = rint(q_i) as floats, in the
// pair layout rr[p] = (element p, element p + 4) of the f32x2 arithmetic.
//
// CORRECTED (16-bit weights): one correction step of the reciprocal product
// (Markstein's division correction), q0 = v * y, r = fma(-q0, s, v),
// q = fma(r, y, q0) with y = RN(1/s).  For every pair of finite 16-bit
// weights v and max m >= |v| whose scale s = fl(m / qmax) (qmax 7 or 127) is
// at least 2^-100, rint(q) equals rint(fl(v / s)) -- checked over all such
// pairs on the GPU, and by test_quant_stream_gpu.py for the kernels -- so
// ties of the quotient are decided like the IEEE quotient's.
//
// Otherwise (fp32 weights): q = v * y, and the sign bits of
// e = fma(d, d, -kNearTie^2), d = q - rint(q), are ANDed into *allneg, which
// stays negative while no quotient is near a tie (one rounding keeps the sign
// of d*d - kNearTie^2).  rint is (q + 1.5*2^23) - 1.5*2^23, round half to even.
template <bool CORRECTED>
__device__ __forceinline__ void quot8(const float (&v)[8], float2 s2, float2 y2, float2 (&rr)[4], int &allneg) {
    const float2 magic2 = make_float2(kRoundMagic, kRoundMagic);
    const float2 nmagic2 = make_float2(-kRoundMagic, -kRoundMagic);
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const float2 w2 = make_float2(v[p], v[p + 4]);
        float2 q = __fmul2_rn(w2, y2);
        if (CORRECTED) q = __ffma2_rn(__ffma2_rn(q, make_float2(-s2.x, -s2.y), w2), y2, q);
        rr[p] = __fadd2_rn(__fadd2_rn(q, magic2), nmagic2);
        if (!CORRECTED) {
            const float2 d = __ffma2_rn(rr[p], make_float2(-1.0f, -1.0f), q);
            const float2 e = __ffma2_rn(d, d, make_float2(-kNearTieSq, -kNearTieSq));
            allneg &= __float_as_int(e.x) & __float_as_int(e.y);
        }
    }
}

// Eight rounded quotients in [-7, 7] -> one word of nibbles (element i in
// bits 4i..4i+3, two's complement).  sum_i (rr_i + 8) * 16^i is formed
// exactly in two 16-bit halves, whose float bit patterns after adding
// 1.5*2^23 carry them in the low bits; XOR 8 per nibble turns the offset-8
// code into two's complement.
__device__ __forceinline__ uint32_t nibbles8(const float2 (&rr)[4]) {
    const float2 c16 = make_float2(16.0f, 16.0f);
    const float2 lo = __ffma2_rn(rr[1], c16, rr[0]);  // (q0 + 16 q1, q4 + 16 q5)
    const float2 hi = __ffma2_rn(rr[3], c16, rr[2]);  // (q2 + 16 q3, q6 + 16 q7)
    const float off = kRoundMagic + 34952.0f;         // 1.5*2^23 + 0x8888
    const float2 h = __fadd2_rn(__ffma2_rn(hi, make_float2(256.0f, 256.0f), lo), make_float2(off, off));
    return __byte_perm(__float_as_uint(h.x), __float_as_uint(h.y), 0x5410) ^ 0x88888888u;
}

// Eight rounded quotients in [-127, 127] -> eight int8 bytes, the same way
// with offset 128 per byte.
__device__ __forceinline__ uint2 bytes8(const float2 (&rr)[4]) {
    const float2 c256 = make_float2(256.0f, 256.0f);
    const float off = kRoundMagic + 32896.0f;  // 1.5*2^23 + 0x8080
    const float2 lo = __fadd2_rn(__ffma2_rn(rr[1], c256, rr[0]), make_float2(off, off));  // elements (0,1), (4,5)
    const float2 hi = __fadd2_rn(__ffma2_rn(rr[3], c256, rr[2]), make_float2(off, off));  // elements (2,3), (6,7)
    return make_uint2(__byte_perm(__float_as_uint(lo.x), __float_as_uint(hi.x), 0x5410) ^ 0x80808080u,
                      __byte_perm(__float_as_uint(lo.y), __float_as_uint(hi.y), 0x5410) ^ 0x80808080u);
}

// fl(m / Q) for m > 0 by the same correction with RN(1/Q); equal to the IEEE
// quotient for every positive finite float m (checked exhaustively on the
// GPU over all 2^31 - 2^23 of them, Q = 7 and 127); scale 1 for m == 0 as
// scale_from_max, NaN / Inf for a non-finite m.
template <int Q> __device__ __forceinline__ float scale_q(float m) {
    constexpr float kInv = 1.0f / (float)Q;
    const float q0 = __fmul_rn(m, kInv);
    const float q = __fmaf_rn(__fmaf_rn(-q0, (float)Q, m), kInv, q0);
    return m == 0.0f ? 1.0f : q;
}

// Does the fast path of quot8 decide every quotient exactly?  16-bit weights:
// for scales in [2^-100, max float]; fp32: for normal scales with no quotient
// near a tie.
template <bool CORRECTED> __device__ __forceinline__ bool quot8_exact(float s, int allneg) {
    if (CORRECTED) return s >= 0x1p-100f && s <= 3.40282347e38f;
    return allneg < 0 && s >= 1.17549435e-38f && s <= 3.40282347e38f;
}

__device__ __forceinline__ uint32_t pack8_exact(const float (&v)[8], float s, float inv) {
    uint32_t word = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) word |= (quant_bits(v[i], s, inv, 7.0f) & 15u) << (4 * i);
    return word;
}

__device__ __forceinline__ uint2 bytes8_exact(const float (&v)[8], float s, float inv) {
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        lo |= (quant_bits(v[i], s, inv, 127.0f) & 0xFFu) << (8 * i);
        hi |= (quant_bits(v[i + 4], s, inv, 127.0f) & 0xFFu) << (8 * i);
    }
    return make_uint2(lo, hi);
}

template <typename T, int G, int CW, int CPT>
__global__ void __launch_bounds__((CW + 1) * 32)
    quant_group_stream_kernel(const T *__restrict__ w, int64_t total, int nstages, uint8_t *__restrict__ packed,
                              float *__restrict__ scales, int32_t *__restrict__ nonfinite) {
    using C = Chunk<T>;
    constexpr int E = kStreamTile / (int)sizeof(T);  // weights per tile
    constexpr int L = G / (8 * CPT);                 // lanes per group
    constexpr int V = CPT * C::kWords / 4;           // 16-byte vectors per thread
    constexpr int VPC = C::kWords / 4;               // vectors per chunk
    constexpr int SLOTS = E / (8 * CPT);
    constexpr int PASSES = SLOTS / (CW * 32);
    static_assert(L >= 1 && L * 8 * CPT == G, "group must split into whole thread shares");
    static_assert(PASSES >= 1 && PASSES * CW * 32 == SLOTS, "tile must split evenly over the consumer threads");
    static_assert(V == 1 || V == 2 || V == 4, "unsupported vectors per thread");
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)nstages * kStreamTile);
    uint64_t *empty = full + nstages;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t tiles = (total + E - 1) / E;
    const int64_t mine = (int64_t)blockIdx.x < tiles ? (tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;

    if (threadIdx.x == 0) {
        for (int i = 0; i < nstages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], CW);
        }
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == CW) {  // ------------------------------------ producer
        if (lane == 0) {
            for (int64_t pos = 0; pos < mine; ++pos) {
                const int slot = (int)(pos % nstages);
                const int64_t round = pos / nstages;
                if (round > 0 && !mbar_wait(&empty[slot], (uint32_t)((round - 1) & 1))) break;
                const int64_t base = ((int64_t)blockIdx.x + pos * gridDim.x) * E;
                const uint32_t bytes = (uint32_t)(min((int64_t)E, total - base) * (int64_t)sizeof(T));
                mbar_arrive_expect_tx(&full[slot], bytes);
                bulk_load_1d(smem + (size_t)slot * kStreamTile, w + base, bytes, &full[slot]);
            }
        }
        return;
    }

    // Vector q of a thread is read from position q ^ x, x = lane bits that
    // put the 8 lanes of a quarter-warp on distinct 16-byte bank groups.
    const int x = V == 1 ? 0 : V == 2 ? (lane >> 2) & 1 : (lane >> 1) & 3;
    const int cx = x / VPC;  // chunk permutation
    const bool halves = VPC == 2 && (x & 1);  // f32: the two halves of every chunk swapped
    bool bad = false;
    for (int64_t pos = 0; pos < mine; ++pos) {
        const int slot = (int)(pos % nstages);
        if (!__all_sync(0xffffffffu, mbar_wait(&full[slot], (uint32_t)((pos / nstages) & 1)))) break;
        const int64_t base = ((int64_t)blockIdx.x + pos * gridDim.x) * E;
        const int valid = (int)min((int64_t)E, total - base);
        const uint8_t *tile = smem + (size_t)slot * kStreamTile;
#pragma unroll
        for (int p = 0; p < PASSES; ++p) {
            const int u = p * CW * 32 + (int)threadIdx.x;
            const int e0 = u * 8 * CPT;
            const bool live = e0 < valid;  // groups lie wholly inside or outside [0, valid)
            uint32_t r[V * 4];
#pragma unroll
            for (int q = 0; q < V; ++q) {
                uint4 t = make_uint4(0, 0, 0, 0);
                if (live) t = *reinterpret_cast<const uint4 *>(tile + (size_t)(u * V + (q ^ x)) * 16);
                r[4 * q] = t.x, r[4 * q + 1] = t.y, r[4 * q + 2] = t.z, r[4 * q + 3] = t.w;
            }
            uint32_t mb = C::absmax(r);
#pragma unroll
            for (int c = 1; c < CPT; ++c) mb = C::combine(mb, C::absmax(r + c * C::kWords));
            mb = C::fold(mb);
#pragma unroll
            for (int o = L / 2; o > 0; o >>= 1) mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, o));
            bad |= mb >= C::kNonFinite;
            const float s = scale_q<7>(C::to_f32(mb));  // NaN / Inf for a non-finite max: exact path
            const float inv = __frcp_rn(s);
            int allneg = -1;
            uint32_t wd[CPT];
#pragma unroll
            for (int c = 0; c < CPT; ++c) {
                float v[8];
                float2 rr[4];
                C::unpack(r + c * C::kWords, v);
                quot8<C::kCorrected>(v, make_float2(s, s), make_float2(inv, inv), rr, allneg);
                wd[c] = nibbles8(rr);
            }
            if (__any_sync(0xffffffffu, !quot8_exact<C::kCorrected>(s, allneg))) {
#pragma unroll
                for (int c = 0; c < CPT; ++c) {
                    float v[8];
                    C::unpack(r + c * C::kWords, v);
                    wd[c] = pack8_exact(v, s, inv);
                }
            }
            if (halves) {
#pragma unroll
                for (int c = 0; c < CPT; ++c) wd[c] = __byte_perm(wd[c], 0, 0x1032);
            }
            // Undo the chunk permutation: word c was computed from chunk c ^ cx.
            if (CPT >= 2 && (cx & 1)) {
#pragma unroll
                for (int c = 0; c < CPT; c += 2) { const uint32_t t = wd[c]; wd[c] = wd[c + 1]; wd[c + 1] = t; }
            }
            if (CPT >= 4 && (cx & 2)) {
#pragma unroll
                for (int c = 0; c < CPT; c += 4) {
                    uint32_t t = wd[c]; wd[c] = wd[c + 2]; wd[c + 2] = t;
                    t = wd[c + 1]; wd[c + 1] = wd[c + 3]; wd[c + 3] = t;
                }
            }
            if (live) {
                uint8_t *dst = packed + (base + e0) / 2;
                if (CPT == 1) *reinterpret_cast<uint32_t *>(dst) = wd[0];
                if (CPT == 2) *reinterpret_cast<uint2 *>(dst) = make_uint2(wd[0], wd[1 % CPT]);
                if (CPT == 4) *reinterpret_cast<uint4 *>(dst) = make_uint4(wd[0], wd[1 % CPT], wd[2 % CPT], wd[3 % CPT]);
                if (lane % L == 0) scales[(base + e0) / G] = s;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
    }
    if (nonfinite != nullptr && bad) *nonfinite = 1;
}

// ------------------------------------------------ streaming per-row quantize --
//
// Per-row INT8 / INT4 (flat packing) for K % 8 == 0: a stage holds R whole
// rows (one 1-D bulk copy of R*K weights), so each weight leaves HBM once.
// All CW consumer warps work on one row at a time: pass 1 reduces the
// integer |w| max from shared memory (warp shuffles, then one named barrier
// over a double-buffered per-warp array), pass 2 quantizes from shared
// memory and stores 8 (INT8) or 4 (INT4) bytes per 8 weights.  With K even,
// row r of the flat INT4 packing is bytes [r*K/2, (r+1)*K/2).
template <typename T, int BITS, int CW>
__global__ void __launch_bounds__((CW + 1) * 32)
    quant_rowwise_stream_kernel(const T *__restrict__ w, int64_t n, int k, int rows_per_stage, int stage_bytes,
                                int nstages, uint8_t *__restrict__ out, float *__restrict__ scales) {
    using C = Chunk<T>;
    constexpr int Q = BITS == 8 ? 127 : 7;
    constexpr int VPC = C::kWords / 4;  // 16-byte vectors per 8-weight chunk
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint32_t red[2][CW];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)nstages * stage_bytes);
    uint64_t *empty = full + nstages;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t stages = (n + rows_per_stage - 1) / rows_per_stage;
    const int64_t mine = (int64_t)blockIdx.x < stages ? (stages - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const size_t row_bytes = (size_t)k * sizeof(T);

    if (threadIdx.x == 0) {
        for (int i = 0; i < nstages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], CW);
        }
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == CW) {  // ------------------------------------ producer
        if (lane == 0) {
            for (int64_t pos = 0; pos < mine; ++pos) {
                const int slot = (int)(pos % nstages);
                const int64_t round = pos / nstages;
                if (round > 0 && !mbar_wait(&empty[slot], (uint32_t)((round - 1) & 1))) break;
                const int64_t row0 = ((int64_t)blockIdx.x + pos * gridDim.x) * rows_per_stage;
                const uint32_t bytes = (uint32_t)(min((int64_t)rows_per_stage, n - row0) * (int64_t)row_bytes);
                mbar_arrive_expect_tx(&full[slot], bytes);
                bulk_load_1d(smem + (size_t)slot * stage_bytes, w + row0 * k, bytes, &full[slot]);
            }
        }
        return;
    }

    // Every consumer warp takes the same number of named barriers (one per
    // row) whatever happens: a warp whose wait fails (an error recorded by any
    // CTA makes later waits return at once) goes on through its rows without
    // storing, so no warp is left waiting at a barrier the others skipped.
    const int chunks = k / 8;
    int parity = 0;
    for (int64_t pos = 0; pos < mine; ++pos) {
        const int slot = (int)(pos % nstages);
        const bool ok = __all_sync(0xffffffffu, mbar_wait(&full[slot], (uint32_t)((pos / nstages) & 1)));
        const int64_t row0 = ((int64_t)blockIdx.x + pos * gridDim.x) * rows_per_stage;
        const int rows = (int)min((int64_t)rows_per_stage, n - row0);
        for (int rr = 0; rr < rows; ++rr) {
            const uint4 *row = reinterpret_cast<const uint4 *>(smem + (size_t)slot * stage_bytes + rr * row_bytes);
            uint32_t mb = 0;
            for (int c = threadIdx.x; c < chunks; c += CW * 32) {
                uint32_t x[C::kWords];
#pragma unroll
                for (int q = 0; q < VPC; ++q) {
                    const uint4 t = row[c * VPC + q];
                    x[4 * q] = t.x, x[4 * q + 1] = t.y, x[4 * q + 2] = t.z, x[4 * q + 3] = t.w;
                }
                mb = C::combine(mb, C::absmax(x));
            }
            mb = C::fold(mb);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, o));
            if (lane == 0) red[parity][warp] = mb;
            asm volatile("bar.sync 1, %0;" ::"r"(CW * 32) : "memory");
#pragma unroll
            for (int i = 0; i < CW; ++i) mb = max(mb, red[parity][i]);
            parity ^= 1;
            const float s = scale_q<Q>(C::to_f32(mb));
            const float inv = __frcp_rn(s);
            const int64_t r = row0 + rr;
            if (ok && threadIdx.x == 0) scales[r] = s;
            const bool slow_row = !quot8_exact<true>(s, -1);  // 16-bit weights: one decision per row
            for (int c = threadIdx.x; c < chunks; c += CW * 32) {
                uint32_t x[C::kWords];
#pragma unroll
                for (int q = 0; q < VPC; ++q) {
                    const uint4 t = row[c * VPC + q];
                    x[4 * q] = t.x, x[4 * q + 1] = t.y, x[4 * q + 2] = t.z, x[4 * q + 3] = t.w;
                }
                float v[8];
                float2 q8[4];
                int allneg = -1;
                C::unpack(x, v);
                quot8<C::kCorrected>(v, make_float2(s, s), make_float2(inv, inv), q8, allneg);
                bool slow = C::kCorrected ? slow_row : !quot8_exact<false>(s, allneg);
                if (!C::kCorrected) slow = __any_sync(__activemask(), slow);
                if (BITS == 8) {
                    const uint2 b = slow ? bytes8_exact(v, s, inv) : bytes8(q8);
                    if (ok) *reinterpret_cast<uint2 *>(out + r * k + 8 * c) = b;
                } else {
                    const uint32_t b = slow ? pack8_exact(v, s, inv) : nibbles8(q8);
                    if (ok) *reinterpret_cast<uint32_t *>(out + r * (k / 2) + 4 * c) = b;
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
    }
}

// Any even group size: one thread per (row, group), scalar loads.
template <typename T>
__global__ void quant_group_generic_kernel(const T *__restrict__ w, int64_t n, int64_t k, int64_t kp, int g,
                                           uint8_t *__restrict__ packed, float *__restrict__ scales,
                                           int32_t *__restrict__ nonfinite) {
    const int64_t groups = kp / g;
    bool bad = false;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n * groups;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = t / groups, gi = t - r * groups;
        const int64_t c0 = gi * g;
        const T *row = w + r * k;
        float mx = 0.0f;
        for (int i = 0; i < g; ++i) {
            const float v = c0 + i < k ? ld(row, c0 + i) : 0.0f;
            bad |= !isfinite(v);
            mx = fmaxf(mx, fabsf(v));
        }
        const float s = scale_from_max(mx, 7.0f);
        const float inv = __frcp_rn(s);
        scales[t] = s;
        uint8_t *dst = packed + r * (kp / 2) + c0 / 2;
        for (int i = 0; i < g; i += 2) {
            const float a = c0 + i < k ? ld(row, c0 + i) : 0.0f;
            const float b = c0 + i + 1 < k ? ld(row, c0 + i + 1) : 0.0f;
            dst[i / 2] = (uint8_t)((quant_bits(a, s, inv, 7.0f) & 15u) | ((quant_bits(b, s, inv, 7.0f) & 15u) << 4));
        }
    }
    if (nonfinite != nullptr && bad) *nonfinite = 1;
}

// ------------------------------------------------------ dequantizers --

__global__ void dequant_int8_kernel(const int8_t *__restrict__ q, const float *__restrict__ scales, int64_t n,
                                    int64_t k, float *__restrict__ out, bool vec) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    if (vec) {  // K % 8 == 0
        const int64_t units = n * k / 8;
        for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < units; u += stride) {
            const int64_t f = 8 * u;
            const float s = scales[f / k];
            const uint2 b = __ldg(reinterpret_cast<const uint2 *>(q + f));
            float o[8];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                o[i] = __fmul_rn((float)(int8_t)(b.x >> (8 * i)), s);
                o[i + 4] = __fmul_rn((float)(int8_t)(b.y >> (8 * i)), s);
            }
            float4 *dst = reinterpret_cast<float4 *>(out + f);
            dst[0] = make_float4(o[0], o[1], o[2], o[3]);
            dst[1] = make_float4(o[4], o[5], o[6], o[7]);
        }
    } else {
        for (int64_t f = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; f < n * k; f += stride)
            out[f] = __fmul_rn((float)q[f], scales[f / k]);
    }
}

__global__ void dequant_int4_row_kernel(const uint8_t *__restrict__ packed, const float *__restrict__ scales,
                                        int64_t n, int64_t k, float *__restrict__ out, bool vec) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t total = n * k;
    if (vec) {  // K % 8 == 0: 8 elements = one aligned 32-bit word, one row
        for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < total / 8; u += stride) {
            const int64_t f = 8 * u;
            const float s = scales[f / k];
            const uint32_t word = __ldg(reinterpret_cast<const uint32_t *>(packed + f / 2));
            float o[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] = __fmul_rn((float)(((int)(word << (28 - 4 * i))) >> 28), s);
            float4 *dst = reinterpret_cast<float4 *>(out + f);
            dst[0] = make_float4(o[0], o[1], o[2], o[3]);
            dst[1] = make_float4(o[4], o[5], o[6], o[7]);
        }
    } else {
        for (int64_t f = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; f < total; f += stride) {
            const int v = nibble_value(packed[f >> 1], (int)(f & 1));
            out[f] = __fmul_rn((float)v, scales[f / k]);
        }
    }
}

__global__ void dequant_int4_group_kernel(const uint8_t *__restrict__ packed, const float *__restrict__ scales,
                                          int64_t n, int64_t k, int64_t kp, int g, float *__restrict__ out,
                                          bool vec) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t groups = kp / g;
    if (vec) {  // K % 8 == 0 and g % 8 == 0: 8 outputs share one scale
        const int64_t per_row = k / 8;
        for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < n * per_row; u += stride) {
            const int64_t r = u / per_row, c = 8 * (u - r * per_row);
            const float s = scales[r * groups + c / g];
            const uint32_t word = __ldg(reinterpret_cast<const uint32_t *>(packed + r * (kp / 2) + c / 2));
            float o[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] = __fmul_rn((float)(((int)(word << (28 - 4 * i))) >> 28), s);
            float4 *dst = reinterpret_cast<float4 *>(out + r * k + c);
            dst[0] = make_float4(o[0], o[1], o[2], o[3]);
            dst[1] = make_float4(o[4], o[5], o[6], o[7]);
        }
    } else {
        for (int64_t f = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; f < n * k; f += stride) {
            const int64_t r = f / k, c = f - r * k;
            const int64_t e = r * kp + c;
            const int v = nibble_value(packed[e >> 1], (int)(e & 1));
            out[f] = __fmul_rn((float)v, scales[r * groups + c / g]);
        }
    }
}

int grid_for(int64_t units, int threads) {
    const int64_t cap = (int64_t)sm_count() * 16;
    int64_t g = cdiv(units, threads);
    if (g > cap) g = cap;
    return (int)(g < 1 ? 1 : g);
}

// Streaming per-row launch; OQ_ERR_UNSUPPORTED when the shape or alignment
// does not qualify (then the two-pass kernel runs).  A stage holds
// floor(16 KB / row bytes) rows (3 stages), or one row of up to 100 KB (2
// stages); as many CTAs per SM as shared memory admits, at most 4.
constexpr int kRowStreamWarps = 8;

template <typename T, int BITS>
int launch_rowwise_stream(const T *w, int64_t n, int64_t k, uint8_t *out, float *scales, cudaStream_t st,
                          int nstages = 0, int ctas_per_sm = 0) {
    if constexpr (std::is_same<T, double>::value) {
        return OQ_ERR_UNSUPPORTED;
    } else {
        const int64_t row_bytes = k * (int64_t)sizeof(T);
        if (k % 8 != 0 || row_bytes > 100 * 1024 || !aligned(w, 16) || !aligned(out, BITS == 8 ? 8 : 4))
            return OQ_ERR_UNSUPPORTED;
        const int rows = (int)std::max<int64_t>(1, std::min<int64_t>(16384 / row_bytes, n));
        const int stage = (int)(((rows * row_bytes) + 127) / 128 * 128);
        if (nstages <= 0) nstages = stage <= 16384 ? 3 : 2;
        const size_t smem = (size_t)nstages * (stage + 16);
        const void *kern = reinterpret_cast<const void *>(&quant_rowwise_stream_kernel<T, BITS, kRowStreamWarps>);
        const int threads = (kRowStreamWarps + 1) * 32;
        const int rc = allow_dynamic_smem(kern, smem);
        if (rc != OQ_OK) return rc;
        if (ctas_per_sm <= 0) {
            OQ_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&ctas_per_sm, kern, threads, smem));
            ctas_per_sm = std::max(1, std::min(4, ctas_per_sm));
        }
        const int64_t grid = std::min<int64_t>(cdiv(n, rows), (int64_t)sm_count() * ctas_per_sm);
        int ki = (int)k;
        void *args[] = {(void *)&w, (void *)&n, (void *)&ki, (void *)&rows, (void *)&stage, (void *)&nstages,
                        (void *)&out, (void *)&scales};
        OQ_CUDA(cudaLaunchKernel(kern, dim3((unsigned)grid), dim3(threads), args, smem, st));
        return OQ_OK;
    }
}

template <typename T, int BITS>
int launch_rowwise(const T *w, int64_t n, int64_t k, uint8_t *out, float *scales, cudaStream_t st) {
    {
        const int rc = launch_rowwise_stream<T, BITS>(w, n, k, out, scales, st);
        if (rc != OQ_ERR_UNSUPPORTED) return rc == OQ_OK ? check_launch("quantize (per-row)") : rc;
    }
    const bool vec = (k % 8 == 0) && aligned(w, 16) && aligned(out, BITS == 8 ? 8 : 4);
    const int64_t units = vec ? k / 8 : k;
    int threads = (int)std::min<int64_t>(kRowThreads, std::max<int64_t>(32, cdiv(units, 32) * 32));
    if (vec)
        quant_rowwise_kernel<T, BITS, true><<<(unsigned)n, threads, 0, st>>>(w, n, k, out, scales);
    else
        quant_rowwise_kernel<T, BITS, false><<<(unsigned)n, threads, 0, st>>>(w, n, k, out, scales);
    if (BITS == 4 && (k & 1) && n > 1)
        straddle_kernel<T><<<grid_for(n, 256), 256, 0, st>>>(w, n, k, out, scales);
    return check_launch("quantize (per-row)");
}

// Streaming quantizer launch for K % g == 0 (g a power of two in [8, 256]),
// 16-byte-aligned weights and 4*CPT-byte-aligned output; returns
// OQ_ERR_UNSUPPORTED when the shape or alignment does not qualify.
constexpr int kStreamWarps = 8;

template <typename T, int CPT>
int launch_group_stream_cpt(const T *w, int64_t total, int g, uint8_t *packed, float *scales, int32_t *flag,
                            int nstages, int ctas_per_sm, cudaStream_t st) {
    constexpr int E = kStreamTile / (int)sizeof(T);
    const int64_t tiles = cdiv(total, E);
    const int64_t grid = std::min<int64_t>(tiles, (int64_t)sm_count() * ctas_per_sm);
    const size_t smem = (size_t)nstages * (kStreamTile + 16);
    const void *kern = nullptr;
    switch (g) {
#define OQ_S(GG)                                                                                          \
    case GG:                                                                                              \
        if constexpr (GG >= 8 * CPT) kern = reinterpret_cast<const void *>(&quant_group_stream_kernel<T, GG, kStreamWarps, CPT>); \
        break;
        OQ_S(8) OQ_S(16) OQ_S(32) OQ_S(64) OQ_S(128) OQ_S(256)
#undef OQ_S
        default: break;
    }
    if (kern == nullptr) return OQ_ERR_UNSUPPORTED;
    const int rc = allow_dynamic_smem(kern, smem);
    if (rc != OQ_OK) return rc;
    void *args[] = {(void *)&w, (void *)&total, (void *)&nstages, (void *)&packed, (void *)&scales, (void *)&flag};
    OQ_CUDA(cudaLaunchKernel(kern, dim3((unsigned)grid), dim3((kStreamWarps + 1) * 32), args, smem, st));
    return OQ_OK;
}

template <typename T>
int launch_group_stream(const T *w, int64_t n, int64_t k, int g, uint8_t *packed, float *scales, int32_t *flag,
                        cudaStream_t st, int nstages = 4, int ctas_per_sm = 3, int cpt = 0) {
    if constexpr (std::is_same<T, double>::value) {
        return OQ_ERR_UNSUPPORTED;
    } else {
        constexpr int kMaxCpt = sizeof(T) == 4 ? 2 : 4;
        if (g < 8 || g > 256 || (g & (g - 1)) != 0 || k % g != 0 || !aligned(w, 16)) return OQ_ERR_UNSUPPORTED;
        if (cpt == 0) cpt = std::min(kMaxCpt, g / 8);  // 16-bit: 32 weights per thread for g >= 32
        if (cpt > kMaxCpt || cpt > g / 8 || !aligned(packed, 4 * cpt)) return OQ_ERR_UNSUPPORTED;
        const int64_t total = n * k;
        if (cpt == 1) return launch_group_stream_cpt<T, 1>(w, total, g, packed, scales, flag, nstages, ctas_per_sm, st);
        if (cpt == 2) return launch_group_stream_cpt<T, 2>(w, total, g, packed, scales, flag, nstages, ctas_per_sm, st);
        if constexpr (kMaxCpt >= 4) {
            if (cpt == 4) return launch_group_stream_cpt<T, 4>(w, total, g, packed, scales, flag, nstages, ctas_per_sm, st);
        }
        return OQ_ERR_UNSUPPORTED;
    }
}

template <typename T>
int launch_group(const T *w, int64_t n, int64_t k, int g, uint8_t *packed, float *scales, int32_t *flag,
                 cudaStream_t st) {
    {
        const int rc = launch_group_stream(w, n, k, g, packed, scales, flag, st);
        if (rc != OQ_ERR_UNSUPPORTED) return rc == OQ_OK ? check_launch("quantize_int4_groupwise") : rc;
    }
    const int64_t kp = cdiv(k, g) * g;
    const bool fast = g >= 8 && g <= 256 && (g & (g - 1)) == 0 && aligned(packed, 4);
    const bool vec = (k % 8 == 0) && aligned(w, 16);
    if (fast) {
        const int64_t units = n * (kp / 8);
        const int threads = 256;
        int64_t blocks = cdiv(units, threads);
        const int64_t cap = (int64_t)sm_count() * 8;
        if (blocks > cap) blocks = cap;
#define OQ_G(LL)                                                                                   \
    case LL:                                                                                       \
        if (vec)                                                                                   \
            quant_group_fast_kernel<T, LL><<<(unsigned)blocks, threads, 0, st>>>(w, n, k, kp, packed, scales, flag); \
        else                                                                                       \
            quant_group_kernel<T, LL, false><<<(unsigned)blocks, threads, 0, st>>>(w, n, k, kp, packed, scales, flag); \
        break;
        switch (g / 8) {
            OQ_G(1) OQ_G(2) OQ_G(4) OQ_G(8) OQ_G(16) OQ_G(32)
        }
#undef OQ_G
    } else {
        const int64_t units = n * (kp / g);
        quant_group_generic_kernel<T><<<grid_for(units, 128), 128, 0, st>>>(w, n, k, kp, g, packed, scales, flag);
    }
    return check_launch("quantize_int4_groupwise");
}

}  // namespace

// Dispatch on the weight dtype.
#define OQ_DISPATCH_DTYPE(dtype, PTR, CALL)                                                       \
    switch (dtype) {                                                                              \
        case OQ_F32: { const float *PTR = static_cast<const float *>(w); return CALL; }           \
        case OQ_F16: { const __half *PTR = static_cast<const __half *>(w); return CALL; }         \
        case OQ_BF16: { const __nv_bfloat16 *PTR = static_cast<const __nv_bfloat16 *>(w); return CALL; } \
        case OQ_F64: { const double *PTR = static_cast<const double *>(w); return CALL; }         \
        default: return invalid("unsupported weight dtype code %d", dtype);                      \
    }

}  // namespace oq

using namespace oq;

extern "C" int oq_quant_int8_rowwise(const void *w, int dtype, int64_t n, int64_t k, int8_t *q, float *scales,
                                     oq_stream_t stream) {
    clear_error();
    OQ_REQUIRE(n >= 1 && k >= 1, "weights must be a nonempty 2-D matrix (got %lld x %lld)", (long long)n, (long long)k);
    OQ_REQUIRE(n < (1ll << 31), "too many rows (%lld)", (long long)n);
    OQ_REQUIRE(w && q && scales, "null pointer argument");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    uint8_t *out = reinterpret_cast<uint8_t *>(q);
    OQ_DISPATCH_DTYPE(dtype, p, (launch_rowwise<std::remove_cv_t<std::remove_pointer_t<decltype(p)>>, 8>(p, n, k, out, scales, st)));
}

extern "C" int oq_quant_int4_rowwise(const void *w, int dtype, int64_t n, int64_t k, uint8_t *packed,
                                     float *scales, oq_stream_t stream) {
    clear_error();
    OQ_REQUIRE(n >= 1 && k >= 1, "weights must be a nonempty 2-D matrix (got %lld x %lld)", (long long)n, (long long)k);
    OQ_REQUIRE(n < (1ll << 31), "too many rows (%lld)", (long long)n);
    OQ_REQUIRE(w && packed && scales, "null pointer argument");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    OQ_DISPATCH_DTYPE(dtype, p, (launch_rowwise<std::remove_cv_t<std::remove_pointer_t<decltype(p)>>, 4>(p, n, k, packed, scales, st)));
}

extern "C" int oq_quant_int4_group(const void *w, int dtype, int64_t n, int64_t k, int group_size,
                                   uint8_t *packed, float *scales, int32_t *nonfinite, oq_stream_t stream) {
    clear_error();
    OQ_REQUIRE(n >= 1 && k >= 1, "Expected nonempty 2D weights (got %lld x %lld)", (long long)n, (long long)k);
    OQ_REQUIRE(group_size >= 2 && group_size % 2 == 0, "Group size must be even and >= 2 (got %d)", group_size);
    OQ_REQUIRE(w && packed && scales, "null pointer argument");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (nonfinite) OQ_CUDA(cudaMemsetAsync(nonfinite, 0, sizeof(int32_t), st));
    OQ_DISPATCH_DTYPE(dtype, p, (launch_group(p, n, k, group_size, packed, scales, nonfinite, st)));
}

extern "C" int oq_dequant_int8_rowwise(const int8_t *q, const float *scales, int64_t n, int64_t k, float *out,
                                       oq_stream_t stream) {
    clear_error();
    OQ_REQUIRE(n >= 1 && k >= 1, "shape must be positive (got %lld x %lld)", (long long)n, (long long)k);
    OQ_REQUIRE(q && scales && out, "null pointer argument");
    const bool vec = k % 8 == 0 && aligned(q, 8) && aligned(out, 16);
    const int64_t units = vec ? n * k / 8 : n * k;
    dequant_int8_kernel<<<grid_for(units, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(q, scales, n, k, out, vec);
    return check_launch("dequantize (INT8)");
}

extern "C" int oq_dequant_int4_rowwise(const uint8_t *packed, const float *scales, int64_t n, int64_t k,
                                       float *out, oq_stream_t stream) {
    clear_error();
    OQ_REQUIRE(n >= 1 && k >= 1, "shape must be positive (got %lld x %lld)", (long long)n, (long long)k);
    OQ_REQUIRE(packed && scales && out, "null pointer argument");
    const bool vec = k % 8 == 0 && aligned(packed, 4) && aligned(out, 16);
    const int64_t units = vec ? n * k / 8 : n * k;
    dequant_int4_row_kernel<<<grid_for(units, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(packed, scales, n, k, out, vec);
    return check_launch("dequantize (INT4)");
}

extern "C" int oq_dequant_int4_group(const uint8_t *packed, const float *scales, int64_t n, int64_t k,
                                     int group_size, float *out, oq_stream_t stream) {
    clear_error();
    OQ_REQUIRE(n >= 1 && k >= 1, "shape must be positive (got %lld x %lld)", (long long)n, (long long)k);
    OQ_REQUIRE(group_size >= 2 && group_size % 2 == 0, "Group size must be even and >= 2 (got %d)", group_size);
    OQ_REQUIRE(packed && scales && out, "null pointer argument");
    const int64_t kp = cdiv(k, group_size) * group_size;
    const bool vec = k % 8 == 0 && group_size % 8 == 0 && aligned(packed, 4) && aligned(out, 16);
    const int64_t units = vec ? n * k / 8 : n * k;
    dequant_int4_group_kernel<<<grid_for(units, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        packed, scales, n, k, kp, group_size, out, vec);
    return check_launch("dequantize_int4_groupwise");
}
