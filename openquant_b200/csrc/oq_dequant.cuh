// Weight dequantization shared by the fused INT4 kernels: the activation
// type traits (packing, legacy mma.sync) and the exact per-weight rounding
// round_x(fl32(q * s)) of openquant/triton_int4.py:62-65.
#pragma once

#include "oq_common.cuh"

namespace oq {

template <typename XT> struct XTraits;
template <> struct XTraits<__half> {
    static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
        __half2 h = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<uint32_t *>(&h);
    }
    static __device__ __forceinline__ float round(float v) { return __half2float(__float2half_rn(v)); }
    static __device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
    static __device__ __forceinline__ __half zero() { return __float2half(0.0f); }
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
    static __device__ __forceinline__ __nv_bfloat16 zero() { return __float2bfloat16(0.0f); }
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
static __device__ __forceinline__ float dq(uint32_t word, int i, float s) {
    const float f = __uint_as_float(0x4B000000u | ((word >> (4 * i)) & 15u));  // 2^23 + u
    return __fmul_rn(__fsub_rn(f, 8388616.0f), s);                               // (u - 8) * s
}

// Per-(row, group) constants of dq_half: s and s * 16^-1 for nibble
// positions 0 and 1, s * 16^-2 and s * 16^-3 for positions 2 and 3, and -8s.
struct DqScale {
    float2 mul01, mul23, m8s;
    float s;
    bool fast;  // s * 16^-3 is a normal float and 8s is finite
};

static __device__ __forceinline__ DqScale make_dq_scale(float s) {
    DqScale d;
    d.s = s;
    d.mul01 = make_float2(s, s * 0.0625f);
    d.mul23 = make_float2(s * 0.00390625f, s * 0.000244140625f);
    d.m8s = make_float2(-8.0f * s, -8.0f * s);
    const float a = fabsf(s);
    d.fast = (a >= 0x1p-100f && a <= 0x1p100f);
    return d;
}

// Four weights -- nibbles 4*H .. 4*H+3 of a packed word (raw two's-complement
// nibbles, element i in bits 4i..4i+3) -> two packed pairs
// {w(2j), w(2j+1)} of round_x(fl32(q * s)).  The word is shifted so the four
// nibbles sit at positions p = 0..3; each is lifted into fp32 as
// 2^23 + u*16^p (u = q + 8, offset binary) by one AND/XOR into the 0x4B000000
// exponent; subtracting 2^23 is exact, and fma(u*16^p, s*16^-p, -8s) is the
// exact value (u - 8) * s = q * s rounded once -- the reference's fp32
// product.  Blackwell's packed f32x2 add/fma do two weights per instruction.
// Scales whose 16^-3 multiple would be subnormal (or non-finite) take the
// per-nibble path.
// (a & b) ^ c in one LOP3 (truth table 0x6A); the compiler otherwise emits
// an AND and an XOR, and the ALU pipe is this kernel's limit.
static __device__ __forceinline__ float and_xor_f(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return __uint_as_float(d);
}

template <typename XT, int H, bool FAST>
static __device__ __forceinline__ void dq_half(uint32_t w, const DqScale &sc, uint32_t (&h)[2]) {
    if (FAST) {
        const uint32_t v = H ? (w >> 16) : w;
        const float f0 = and_xor_f(v, 0x000Fu, 0x4B000008u);
        const float f1 = and_xor_f(v, 0x00F0u, 0x4B000080u);
        const float f2 = and_xor_f(v, 0x0F00u, 0x4B000800u);
        const float f3 = and_xor_f(v, 0xF000u, 0x4B008000u);
        const float2 m23 = make_float2(-8388608.0f, -8388608.0f);
        const float2 w01 = __ffma2_rn(__fadd2_rn(make_float2(f0, f1), m23), sc.mul01, sc.m8s);
        const float2 w23 = __ffma2_rn(__fadd2_rn(make_float2(f2, f3), m23), sc.mul23, sc.m8s);
        h[0] = XTraits<XT>::pack(w01.x, w01.y);
        h[1] = XTraits<XT>::pack(w23.x, w23.y);
    } else {
        const uint32_t u = w ^ 0x88888888u;
        h[0] = XTraits<XT>::pack(dq(u, 4 * H, sc.s), dq(u, 4 * H + 1, sc.s));
        h[1] = XTraits<XT>::pack(dq(u, 4 * H + 2, sc.s), dq(u, 4 * H + 3, sc.s));
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
// cover M <= 8*NT.
//
// The inner loop carries no bounds logic: rows past N are clamped to row N-1
// (their outputs are never stored), prefetches past the last chunk are
// clamped to it, lane segments past KP read column 0 with a zero scale, and
// x is either staged in shared memory zero-padded to 128*nchunks columns
// (XS) or, when it is too large, read from global memory (then KP == K and
// KP % 128 == 0 are required).  Batch lanes >= M keep zero B fragments via
// predicated loads into registers zeroed once.

}  // namespace oq
