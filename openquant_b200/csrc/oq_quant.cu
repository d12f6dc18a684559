// Quantize and dequantize kernels: per-row INT8, per-row flat-packed INT4 and
// groupwise INT4 (openquant 0.5.0 formats), sm_100a.
//
// All of these are HBM-streaming kernels: 16-byte vector loads of 8
// consecutive weights per thread, warp-shuffle max reductions, 4-/8-byte
// packed stores.  Bit-exactness with the reference rests on oq::quant_bits()
// (IEEE quotient, round-half-even) and oq::scale_from_max() (IEEE division).
#include "oq_common.cuh"

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

// Eight quotients q_i = clip(rint(fl(v_i / s)), -qmax, qmax) as the bit
// patterns of (q_i + 1.5*2^23) (low byte / nibble = q_i), like quant_bits but
// with packed f32x2 arithmetic: r = v * (1/s), t = r + 1.5*2^23 (round half
// to even), d = r - (t - 1.5*2^23).  When any lane of `mask` has a quotient
// within 1e-3 of a tie (|d| >= 0.499) or a scale that is not a normal float
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
        slow |= !(fabsf(d.x) < 0.499f) | !(fabsf(d.y) < 0.499f);
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

template <typename T, int BITS>
int launch_rowwise(const T *w, int64_t n, int64_t k, uint8_t *out, float *scales, cudaStream_t st) {
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

template <typename T>
int launch_group(const T *w, int64_t n, int64_t k, int g, uint8_t *packed, float *scales, int32_t *flag,
                 cudaStream_t st) {
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
