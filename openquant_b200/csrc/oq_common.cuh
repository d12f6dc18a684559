// Shared helpers of the openquant_b200 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <string>
#include <type_traits>

#include "../../include/openquant_b200.h"

namespace oq {

// ---------------------------------------------------------------- errors --

void set_error(const char *fmt, ...);
void clear_error();

// Returns OQ_ERR_INVALID with a message.
int invalid(const char *fmt, ...);

// Checks the launch status of the kernels just enqueued.
int check_launch(const char *what);

#define OQ_REQUIRE(cond, ...)                                                    \
    do {                                                                         \
        if (!(cond)) return ::oq::invalid(__VA_ARGS__);                          \
    } while (0)

#define OQ_CUDA(call)                                                            \
    do {                                                                         \
        cudaError_t err_ = (call);                                               \
        if (err_ != cudaSuccess) {                                               \
            ::oq::set_error("%s failed: %s", #call, cudaGetErrorString(err_));   \
            return OQ_ERR_CUDA;                                                  \
        }                                                                        \
    } while (0)

inline bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

inline int dtype_size(int dtype) {
    switch (dtype) {
        case OQ_F32: return 4;
        case OQ_F16: return 2;
        case OQ_BF16: return 2;
        case OQ_F64: return 8;
        default: return 0;
    }
}

// Most GPUs one sharded output is written to (this one and its peers).
constexpr int kMaxOutGpus = 8;

// Output of a linear layer: y[b][feature] as fp32, fp16 or bf16 (OQ_F32 /
// OQ_F16 / OQ_BF16), with an optional fp32 bias per output feature added in
// fp32 before the single rounding to the output type.  Element (b, f) goes
// to y[b * ld + col0 + f] -- ld = the layer's N and col0 = 0 for a plain
// layer; for an N-column shard, ld is the full layer's N and col0 the
// shard's first column -- and, for a shard, to the same element of each
// peer GPU's output (npeers buffers mapped over NVLink, plain stores).
struct OutSpec {
    void *y;
    const float *bias;  // nullptr: no bias
    int dtype;
    int npeers = 0;
    int64_t ld = 0;
    int64_t col0 = 0;
    void *peer[kMaxOutGpus - 1] = {};

    template <typename T>
    __device__ __forceinline__ void put(T v, size_t idx) const {
        static_cast<T *>(y)[idx] = v;
#pragma unroll
        for (int p = 0; p < kMaxOutGpus - 1; ++p)  // constant indices: the pointers stay in the parameter bank
            if (p < npeers) static_cast<T *>(peer[p])[idx] = v;
    }
    __device__ __forceinline__ void store(int64_t b, int feature, float v) const {
        if (bias != nullptr) v += __ldg(bias + feature);
        const size_t idx = (size_t)(b * ld + col0 + feature);
        if (dtype == OQ_F16)
            put(__float2half_rn(v), idx);
        else if (dtype == OQ_BF16)
            put(__float2bfloat16_rn(v), idx);
        else
            put(v, idx);
    }
    // Stores v[j] (fp32 bit patterns) as batch rows b0 + j < bend of one
    // feature: a GEMM epilogue's column of the accumulator.  Converts once,
    // then writes the run to each destination in turn (one GPU's stores
    // back to back).
    template <int CNT>
    __device__ __forceinline__ void store_run(int64_t b0, int64_t bend, int feature, const uint32_t (&v)[CNT]) const {
        const int64_t off = b0 * ld + col0 + feature;
        const int64_t cnt = bend - b0;
        float bv = 0.0f;
        if (bias != nullptr) bv = __ldg(bias + feature);
        if (dtype == OQ_F16)
            put_run<__half>(off, cnt, v, bv);
        else if (dtype == OQ_BF16)
            put_run<__nv_bfloat16>(off, cnt, v, bv);
        else
            put_run<float>(off, cnt, v, bv);
    }
    template <typename T, int CNT>
    __device__ __forceinline__ void put_run(int64_t off, int64_t cnt, const uint32_t (&v)[CNT], float bv) const {
        T vals[CNT];
#pragma unroll
        for (int j = 0; j < CNT; ++j) {
            float f = __uint_as_float(v[j]);
            if (bias != nullptr) f += bv;  // no bias: no add (it would turn -0 into +0)
            if constexpr (std::is_same<T, __half>::value)
                vals[j] = __float2half_rn(f);
            else if constexpr (std::is_same<T, __nv_bfloat16>::value)
                vals[j] = __float2bfloat16_rn(f);
            else
                vals[j] = f;
        }
#pragma unroll
        for (int d = 0; d < kMaxOutGpus; ++d) {
            if (d > npeers) break;
            T *dst = static_cast<T *>(d == 0 ? y : peer[d > 0 ? d - 1 : 0]) + off;
            if (cnt >= CNT) {
#pragma unroll
                for (int j = 0; j < CNT; ++j) dst[j * ld] = vals[j];
            } else {
#pragma unroll
                for (int j = 0; j < CNT; ++j)
                    if (j < cnt) dst[j * ld] = vals[j];
            }
        }
    }
};

// Number of SMs of the current device (cached per device).
int sm_count();
// Raises a kernel's dynamic shared-memory limit to `bytes` on the current
// device (once per kernel, device and size; thread-safe).
int allow_dynamic_smem(const void *kern, size_t bytes);

__host__ __device__ inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// ------------------------------------------------------- element loading --

template <typename T> struct Elem;
template <> struct Elem<float> {
    static __device__ __forceinline__ float to_f32(float v) { return v; }
};
template <> struct Elem<__half> {
    static __device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
};
template <> struct Elem<__nv_bfloat16> {
    static __device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
};
template <> struct Elem<double> {
    // np.asarray(..., dtype=np.float32) rounds to nearest even.
    static __device__ __forceinline__ float to_f32(double v) { return __double2float_rn(v); }
};

// Loads 8 consecutive elements starting at p (16-byte aligned for 2-byte
// types, 32-byte for fp32, 64-byte for fp64) and widens them to fp32.
template <typename T> __device__ __forceinline__ void load8(const T *p, float (&v)[8]);

template <> __device__ __forceinline__ void load8<float>(const float *p, float (&v)[8]) {
    float4 a = __ldg(reinterpret_cast<const float4 *>(p));
    float4 b = __ldg(reinterpret_cast<const float4 *>(p) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
template <> __device__ __forceinline__ void load8<__half>(const __half *p, float (&v)[8]) {
    uint4 a = __ldg(reinterpret_cast<const uint4 *>(p));
    const __half2 *h = reinterpret_cast<const __half2 *>(&a);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 f = __half22float2(h[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
    }
}
template <> __device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16 *p, float (&v)[8]) {
    uint4 a = __ldg(reinterpret_cast<const uint4 *>(p));
    // bf16 -> fp32 is a 16-bit left shift of the pattern.
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        v[2 * i] = __uint_as_float(w[i] << 16);
        v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
}
template <> __device__ __forceinline__ void load8<double>(const double *p, float (&v)[8]) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        double2 d = __ldg(reinterpret_cast<const double2 *>(p) + i);
        v[2 * i] = __double2float_rn(d.x);
        v[2 * i + 1] = __double2float_rn(d.y);
    }
}

// -------------------------------------------------------- quantization --

// 1.5 * 2^23: adding it to |v| < 2^22 rounds v to an integer (ties to
// even, the default rounding mode) and leaves that integer, in two's
// complement, in the low mantissa bits of the sum.
constexpr float kRoundMagic = 12582912.0f;

// q = clip(rint(fl(w / s)), -qmax, qmax) with fl() the IEEE-754 fp32
// quotient, returned as the bit pattern of (q + 1.5*2^23): the low byte is
// q as int8, the low nibble is q as a two's-complement int4.  NaN quotients
// give 0 (what the reference's float->int8 cast yields for them).
//
// Fast path: r = w * (1/s) differs from the IEEE quotient by at most
// 3 * 2^-24 * |w/s| <= 2.3e-5 here (|w/s| <= 127 * (1 + 2^-22)), so when r
// is farther than 0.001 from a half-integer both round to the same integer.
// Quotients near a tie, outside [-qmax, qmax], or non-finite take the exact
// path (__fdiv_rn, IEEE round-to-nearest division).
__device__ __forceinline__ uint32_t quant_bits(float w, float s, float inv_s, float qmax) {
    float r = __fmul_rn(w, inv_s);
    float t = __fadd_rn(r, kRoundMagic);
    float rr = __fsub_rn(t, kRoundMagic);
    float d = __fsub_rn(r, rr);
    if (!(fabsf(d) < 0.499f && fabsf(rr) <= qmax)) {
        float e = __fdiv_rn(w, s);
        // NaN first: fmaxf/fminf would turn a NaN into -qmax.
        e = (e != e) ? 0.0f : fminf(fmaxf(rintf(e), -qmax), qmax);
        t = __fadd_rn(e, kRoundMagic);
    }
    return __float_as_uint(t);
}

// scale = max / qmax (IEEE division), 1.0 when max == 0.  A NaN max (a NaN
// in the row) propagates, as np.max does.
__device__ __forceinline__ float scale_from_max(float mx, float qmax) {
    return (mx == 0.0f) ? 1.0f : __fdiv_rn(mx, qmax);
}

// |v| max that propagates NaN (np.max semantics).
__device__ __forceinline__ float nan_max(float a, float b) {
    return (a != a || b != b) ? __int_as_float(0x7fffffff) : fmaxf(a, b);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = nan_max(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Signed value of nibble `i` (0 = low) of a packed byte.
__device__ __forceinline__ int nibble_value(uint32_t byte, int i) {
    int u = (byte >> (4 * i)) & 15;
    return u >= 8 ? u - 16 : u;
}

}  // namespace oq
