// INT8 x INT8 GEMM on the 5th-generation tensor cores (tcgen05.mma
// kind::i8, int32 accumulators in TMEM), sm_100a: the W8A8 linear layer.
//
// y[M][N] = sx[m] * sw[n] * sum_k qx[m][k] * qw[n][k], with qx / sx the
// per-token INT8 quantization of the activations and qw / sw the per-row INT8
// weights -- both exactly the reference's quantize(bits=8) format
// (openquant/quantization.py:14-40), int8 data and one fp32 scale per row.
// The integer products are summed exactly in int32; the result is converted
// to fp32 and multiplied by the two scales.
//
// As in the INT4 GEMM the product is computed transposed, D = W . X^T:
//   tile      : 128 weight rows (MMA M = TMEM lanes) x 256 batch rows (MMA N)
//   k-block   : 128 int8 columns (one 128-byte swizzle atom)
//   producer  : warp 0 -- TMA of the weight tile (128 x 128 B) and of the x
//               tile (256 x 128 B), both 128-byte swizzled, into a 4-stage
//               shared-memory ring (full[s])
//   MMA       : warp 1, one thread -- four tcgen05.mma kind::i8 (K = 32) per
//               k-block, both operands from shared memory by descriptor,
//               into one of two TMEM accumulators (2 x 256 int32 columns);
//               tcgen05.commit frees the stage (empty[s]) and publishes a
//               finished tile (acc_full[b])
//   epilogue  : warps 4..7 -- tcgen05.ld of the accumulator, scaling, fp32
//               stores (32 consecutive weight rows of one batch row per warp
//               store), then acc_empty[b]; the next tile's MMAs run into the
//               other accumulator meanwhile
//   warp 2    : TMEM allocation / release (512 columns)
//
// The grid is persistent (one CTA per SM), tiles ordered so that CTAs on one
// weight tile run together.  Every mbarrier wait is bounded (oq_sm100.cuh);
// on a timeout the roles drain what they have in flight and the kernel
// returns with the device error word set.
#include "oq_sm100.cuh"

#include <algorithm>
#include <mutex>
#include <utility>
#include <vector>

namespace oq {
namespace {

constexpr int kI8BN = 128;                 // weight rows per tile (MMA M, TMEM lanes)
constexpr int kI8BX = 256;                 // batch rows per tile (MMA N)
constexpr int kI8BK = 128;                 // int8 columns per k-block (128 bytes)
constexpr int kI8Stages = 4;
constexpr int kI8WBytes = kI8BN * kI8BK;   // 16 KB weight tile per stage
constexpr int kI8XBytes = kI8BX * kI8BK;   // 32 KB x tile per stage
constexpr int kI8AccCols = kI8BX;          // int32 accumulator columns (one buffer)
constexpr int kI8TmemCols = 2 * kI8AccCols;
constexpr int kI8Threads = 256;            // 8 warps (warp 3 idle)
constexpr size_t kI8Smem = 1024 + (size_t)kI8Stages * (kI8WBytes + kI8XBytes) + 256;

// Instruction descriptor of tcgen05.mma kind::i8: s32 accumulate, A and B
// signed 8-bit, both K-major (same field layout as kind::f16).
__host__ __device__ constexpr uint32_t umma_idesc_s8(int m, int n) {
    return (2u << 4)                       // D format: s32
           | (1u << 7)                     // A format: signed 8-bit
           | (1u << 10)                    // B format: signed 8-bit
           | ((uint32_t)(n >> 3) << 17)    // N / 8
           | ((uint32_t)(m >> 4) << 24);   // M / 16
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::i8.
__device__ __forceinline__ void tc_mma_ss_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__global__ void __launch_bounds__(kI8Threads, 1)
    gemm_w8a8_tcgen05_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                             const float *__restrict__ sx, const float *__restrict__ sw, float *__restrict__ y, int m,
                             int n, int k) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    uint8_t *xbuf = smem;                                       // [S][256 rows][128 B], swizzled
    uint8_t *wbuf = xbuf + (size_t)kI8Stages * kI8XBytes;       // [S][128 rows][128 B], swizzled
    uint64_t *full = reinterpret_cast<uint64_t *>(wbuf + (size_t)kI8Stages * kI8WBytes);
    uint64_t *empty = full + kI8Stages;
    uint64_t *acc_full = empty + kI8Stages;   // [2]
    uint64_t *acc_empty = acc_full + 2;       // [2]
    uint64_t *mma_done = acc_empty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma_done + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles_n = (n + kI8BN - 1) / kI8BN, tiles_m = (m + kI8BX - 1) / kI8BX;
    const int tiles = tiles_n * tiles_m;
    const int kblocks = (k + kI8BK - 1) / kI8BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kI8Stages; ++s) {
            mbar_init(&full[s], 1);   // producer's expect_tx arrival
            mbar_init(&empty[s], 1);  // tcgen05.commit
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);   // tcgen05.commit
            mbar_init(&acc_empty[b], 4);  // one arrival per epilogue warp
        }
        mbar_init(mma_done, 1);
        fence_barrier_init();
    }
    if (warp == 2) {
        tmem_alloc(tmem_slot, kI8TmemCols);
        tmem_relinquish();
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");

    if (warp == 0) {
        // ------------------------------------------------------ producer
        if (lane == 0) {
            tma_prefetch_desc(&xmap);
            tma_prefetch_desc(&wmap);
            int it = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
                const int n0 = (tile / tiles_m) * kI8BN, m0 = (tile % tiles_m) * kI8BX;
                for (int kb = 0; kb < kblocks; ++kb, ++it) {
                    const int s = it % kI8Stages, r = it / kI8Stages;
                    if (r > 0 && !(ok = mbar_wait(&empty[s], (r - 1) & 1))) break;
                    mbar_arrive_expect_tx(&full[s], kI8XBytes + kI8WBytes);
                    tma_load_2d(xbuf + (size_t)s * kI8XBytes, &xmap, &full[s], kb * kI8BK, m0);
                    tma_load_2d(wbuf + (size_t)s * kI8WBytes, &wmap, &full[s], kb * kI8BK, n0);
                }
            }
            // Drain: every issued stage's copies must land before the CTA
            // exits (normally the MMA thread has waited for all of them).
            for (int j = (it > kI8Stages ? it - kI8Stages : 0); j < it; ++j)
                mbar_wait(&full[j % kI8Stages], (j / kI8Stages) & 1);
        }
    } else if (warp == 1) {
        // ----------------------------------------------------------- MMA
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_s8(kI8BN, kI8BX);
            int it = 0, ti = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++ti) {
                const int b = ti & 1;
                if (ti >= 2 && !(ok = mbar_wait(&acc_empty[b], ((ti >> 1) - 1) & 1))) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem + b * kI8AccCols;
                for (int kb = 0; kb < kblocks; ++kb, ++it) {
                    const int s = it % kI8Stages, r = it / kI8Stages;
                    if (!(ok = mbar_wait(&full[s], r & 1))) break;
                    tc_fence_after();
                    const uint64_t adesc = umma_desc_sw128(smem_u32(wbuf + (size_t)s * kI8WBytes));
                    const uint64_t bdesc = umma_desc_sw128(smem_u32(xbuf + (size_t)s * kI8XBytes));
#pragma unroll
                    for (int kk = 0; kk < kI8BK / 32; ++kk)  // K = 32 bytes per MMA: +2 in 16-byte units
                        tc_mma_ss_i8(d_tmem, adesc + (uint64_t)(kk * 2), bdesc + (uint64_t)(kk * 2), idesc,
                                     (kb | kk) != 0 ? 1u : 0u);
                    tc_commit(&empty[s]);
                }
                if (ok) tc_commit(&acc_full[b]);
            }
            // Every MMA this thread issued has completed once mma_done fires.
            tc_commit(mma_done);
            mbar_wait(mma_done, 0);
        }
    } else if (warp >= 4) {
        // ------------------------------------------------------ epilogue
        const int q = warp - 4;  // TMEM lane quarter
        int ti = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++ti) {
            const int b = ti & 1;
            const int n0 = (tile / tiles_m) * kI8BN, m0 = (tile % tiles_m) * kI8BX;
            // Warp-uniform outcome: tcgen05.ld is .sync.aligned.
            ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[b], (ti >> 1) & 1));
            if (!ok) break;
            tc_fence_after();
            const int row = n0 + q * 32 + lane;
            const float swr = row < n ? __ldg(sw + row) : 0.0f;
#pragma unroll 1
            for (int c = 0; c < kI8AccCols / 32; ++c) {
                uint32_t v[32];
                tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + b * kI8AccCols + c * 32, v);
                tc_wait_ld();
                if (row < n) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const int mb = m0 + c * 32 + j;
                        if (mb < m) y[(size_t)mb * n + row] = (float)(int)v[j] * swr * __ldg(sx + mb);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[b]);
        }
    }

    // Lane 0 of warps 0 and 1 ran their roles alone: converge each warp
    // before the CTA-wide barrier (an aligned barrier in a diverged warp is
    // undefined), so that TMEM is released only after every role is done.
    __syncwarp();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem, kI8TmemCols);
    }
}

}  // namespace

// The W8A8 GEMM takes: K % 16 == 0 (16-byte rows for TMA), 16-byte aligned
// qx and qw, sizes below 2^31.
int gemm_w8a8_supported(int64_t m, int64_t n, int64_t k, const int8_t *qx, const int8_t *qw) {
    if (m < 1 || n < 1 || k < 1 || k % 16 != 0) return 0;
    if (!aligned(qx, 16) || !aligned(qw, 16)) return 0;
    if (m >= (1ll << 31) || n >= (1ll << 31) || k >= (1ll << 31) || m * n >= (1ll << 40)) return 0;
    return 1;
}

int gemm_w8a8_launch(const int8_t *qx, const float *sx, const int8_t *qw, const float *sw, float *y, int64_t m,
                     int64_t n, int64_t k, cudaStream_t st) {
    CUtensorMap xmap, wmap;
    int rc = make_tensor_map_2d(&xmap, qx, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)k, (uint64_t)m, (uint64_t)k,
                                kI8BK, kI8BX, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != OQ_OK) return rc;
    rc = make_tensor_map_2d(&wmap, qw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)k, (uint64_t)n, (uint64_t)k, kI8BK,
                            kI8BN, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != OQ_OK) return rc;
    const void *kern = reinterpret_cast<const void *>(&gemm_w8a8_tcgen05_kernel);
    rc = allow_dynamic_smem(kern, kI8Smem);
    if (rc != OQ_OK) return rc;
    const int64_t tiles = cdiv(n, kI8BN) * cdiv(m, kI8BX);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)std::min<int64_t>(tiles, sm_count()));
    cfg.blockDim = dim3(kI8Threads);
    cfg.dynamicSmemBytes = kI8Smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t err = cudaLaunchKernelEx(&cfg, gemm_w8a8_tcgen05_kernel, xmap, wmap, sx, sw, y, (int)m, (int)n, (int)k);
    if (err != cudaSuccess) {
        set_error("int8 GEMM (tcgen05): launch failed: %s", cudaGetErrorString(err));
        return OQ_ERR_CUDA;
    }
    return OQ_OK;
}

}  // namespace oq

using namespace oq;

extern "C" int oq_int8_gemm(const int8_t *qx, const float *sx, const int8_t *qw, const float *sw, float *y,
                            int64_t m, int64_t n, int64_t k, oq_stream_t stream) {
    clear_error();
    OQ_REQUIRE(m >= 1 && n >= 1 && k >= 1, "Matrix dimensions must be positive");
    OQ_REQUIRE(qx && sx && qw && sw && y, "null pointer argument");
    OQ_REQUIRE(k % 16 == 0, "K must be a multiple of 16 (16-byte rows), got %lld", (long long)k);
    OQ_REQUIRE(aligned(qx, 16) && aligned(qw, 16), "int8 operands must be 16-byte aligned");
    OQ_REQUIRE(gemm_w8a8_supported(m, n, k, qx, qw), "shape too large for the INT8 GEMM");
    const int rc = gemm_w8a8_launch(qx, sx, qw, sw, y, m, n, k, static_cast<cudaStream_t>(stream));
    return rc == OQ_OK ? check_launch("int8 GEMM") : rc;
}

// ------------------------------------------------ W8A8 without allocation --
//
// oq_int8_linear_noalloc runs the whole W8A8 layer -- per-token INT8
// quantization of x, then the INT8 GEMM -- for callers that cannot allocate
// device memory when they call in: a host runtime that lends the library only
// the tensors it owns and has no allocator hook to offer, or a service whose
// device memory is fixed at start-up.  The layer's intermediate data (the
// int8 activations and their per-token scales) lives in the fixed array
// below, which the library's module holds on every GPU that loads it, until
// the process exits.  Limits: M * K <= 16 MiB of int8 activations and
// M <= 16384 tokens.
namespace {

constexpr int64_t kNoAllocQxBytes = int64_t(16) << 20;  // int8 activations, M * K
constexpr int64_t kNoAllocRows = 16384;                 // per-token fp32 scales

// [0, 16 MiB): qx [M][K] int8; [16 MiB, +64 KiB): sx [M] fp32.
static __device__ __align__(256) uint8_t g_w8a8_scratch[kNoAllocQxBytes + kNoAllocRows * 4];

std::mutex g_scratch_mutex;
// Resolved addresses, one per CUDA context: a device can carry more than one
// context (a primary one and ones made with cuCtxCreate), and the array has
// a different address in each.
std::vector<std::pair<CUcontext, void *>> g_scratch_address;

CUresult current_context(CUcontext *ctx) {
    static PFN_cuCtxGetCurrent_v4000 get = nullptr;
    if (get == nullptr) {
        cudaDriverEntryPointQueryResult q;
        void *fn = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || fn == nullptr)
            return CUDA_ERROR_NOT_FOUND;
        get = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(fn);
    }
    return get(ctx);
}

// Device address of g_w8a8_scratch in the current context.  Host code only
// sees a host-side stand-in under that name, so the address is looked up
// once per context (cudaGetSymbolAddress, with that context current) and
// kept.  A context destroyed and made again (cudaDeviceReset) can come back
// under the same handle with the array elsewhere, which this cache cannot
// tell: the entry point is not for processes that reset a device.
int scratch_address(void **out) {
    int dev = -1;
    OQ_CUDA(cudaGetDevice(&dev));
    OQ_CUDA(cudaSetDevice(dev));  // the same device: makes its primary context current if none is
    CUcontext ctx = nullptr;
    if (current_context(&ctx) != CUDA_SUCCESS || ctx == nullptr) {
        set_error("int8 linear (no-alloc): no current CUDA context on device %d", dev);
        return OQ_ERR_CUDA;
    }
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    for (const auto &e : g_scratch_address)
        if (e.first == ctx) {
            *out = e.second;
            return OQ_OK;
        }
    void *p = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&p, g_w8a8_scratch);
    if (err != cudaSuccess || p == nullptr) {
        set_error("int8 linear (no-alloc): cannot resolve the scratch array on device %d: %s", dev,
                  cudaGetErrorString(err));
        return OQ_ERR_CUDA;
    }
    g_scratch_address.emplace_back(ctx, p);
    *out = p;
    return OQ_OK;
}

}  // namespace

extern "C" int oq_int8_linear_noalloc(const void *x, int x_dtype, const int8_t *qw, const float *sw, float *y,
                                      int64_t m, int64_t n, int64_t k, oq_stream_t stream) {
    clear_error();
    OQ_REQUIRE(m >= 1 && n >= 1 && k >= 1, "Matrix dimensions must be positive");
    OQ_REQUIRE(x && qw && sw && y, "null pointer argument");
    OQ_REQUIRE(x_dtype == OQ_F32 || x_dtype == OQ_F16 || x_dtype == OQ_BF16, "x must be fp32, fp16 or bf16");
    OQ_REQUIRE(k % 16 == 0, "K must be a multiple of 16 (16-byte rows), got %lld", (long long)k);
    OQ_REQUIRE(aligned(qw, 16), "int8 weights must be 16-byte aligned");
    OQ_REQUIRE(m <= kNoAllocRows && m * k <= kNoAllocQxBytes,
               "int8 linear (no-alloc): M = %lld, K = %lld exceed the fixed scratch (M <= %lld and M * K <= %lld)",
               (long long)m, (long long)k, (long long)kNoAllocRows, (long long)kNoAllocQxBytes);
    void *base = nullptr;
    int rc = scratch_address(&base);
    if (rc != OQ_OK) return rc;
    int8_t *qx = static_cast<int8_t *>(base);
    float *sx = reinterpret_cast<float *>(static_cast<uint8_t *>(base) + kNoAllocQxBytes);
    OQ_REQUIRE(gemm_w8a8_supported(m, n, k, qx, qw), "shape too large for the INT8 GEMM");
    // Every byte of qx[M][K] and sx[M] that the GEMM reads is written by the
    // quantizer first (rows past M come from TMA's zero fill), so nothing in
    // the array needs clearing between calls.
    rc = oq_quant_int8_rowwise(x, x_dtype, m, k, qx, sx, stream);
    if (rc != OQ_OK) return rc;
    rc = gemm_w8a8_launch(qx, sx, qw, sw, y, m, n, k, static_cast<cudaStream_t>(stream));
    return rc == OQ_OK ? check_launch("int8 linear (no-alloc)") : rc;
}
