// Prefill-side fused INT4 dequant + GEMM on the 5th-generation tensor cores
// (tcgen05 / TMEM), sm_100a.
//
// y[M][N] = x[M][K] . W^T with W[n][k] = round_x(fl32(q * s)) exactly as the
// reference kernel rounds its weights (openquant/triton_int4.py:62-65), fp32
// accumulation.  The product is computed transposed, D = W . x^T, so that the
// dequantized weights can be the MMA's A operand held in tensor memory:
//
//   tile      : 128 weight rows (MMA M = TMEM lanes) x 256 batch rows (MMA N)
//   k-block   : 64 columns (one 128-byte swizzle atom of 16-bit x)
//   producer  : warp 0 -- TMA of the x tile (256 x 64, 128-byte swizzle) and
//               of the packed weight tile (128 rows x 32 bytes) per k-block
//               into a 4-stage shared-memory ring (full[s])
//   dequant   : warps 8..8+4*kDqSplit-1 -- warp 8 + 4p + q serves TMEM
//               lane quarter q: its thread for weight row r reads part p of
//               the row's 32 packed bytes, forms the exactly-rounded 16-bit
//               weights and writes them straight into the stage's TMEM A slot
//               with tcgen05.st (no shared-memory round trip), then signals
//               deq[s]; several warps per quarter hide the dequant latency
//   MMA       : warp 1, one thread -- four tcgen05.mma (K = 16 each) per
//               k-block, A from TMEM, B (x) from shared memory by descriptor,
//               D (128 x 256 fp32) accumulating in TMEM; tcgen05.commit frees
//               the stage (empty[s]) and, after the last k-block, publishes
//               the tile (acc_full)
//   epilogue  : warps 4..7 -- tcgen05.ld of the accumulator, fp32 stores
//               (each warp store is 32 consecutive weight rows of one batch
//               row: 128 coalesced bytes), then acc_empty
//   warp 2    : TMEM allocation / release (512 columns: accumulator 256 +
//               4 A slots of 32)
//
// The grid is persistent (one CTA per SM); tiles are ordered so that the
// CTAs working on one weight tile run together, so each packed weight tile
// is read from HBM once while x stays resident in L2.  Every mbarrier wait
// is bounded (oq_sm100.cuh); on a timeout the roles drain what they have in
// flight and the kernel returns with the device error word set.
#include "oq_dequant.cuh"
#include "oq_sm100.cuh"

#include <mutex>
#include <set>

namespace oq {
namespace {

constexpr int kBN = 128;                 // weight rows per tile (MMA M, TMEM lanes)
constexpr int kBX = 256;                 // batch rows per tile (MMA N)
constexpr int kBK = 64;                  // columns per k-block
constexpr int kStages = 4;
constexpr int kXBytes = kBX * kBK * 2;   // 32 KB x tile per stage
constexpr int kWBytes = kBN * kBK / 2;   // 4 KB packed tile per stage
constexpr int kAccCols = kBX;            // fp32 accumulator columns
constexpr int kACols = kBK / 2;          // TMEM columns of one A slot (two 16-bit values per column)
constexpr int kTmemCols = 512;
// Dequant warps per TMEM lane quarter: each fills 64 / kDqSplit columns of a
// k-block, so one k-block is spread over 4 * kDqSplit warps.
constexpr int kDqSplit = 1;
constexpr int kDqWords = 8 / kDqSplit;   // packed words per dequant thread per k-block
constexpr int kThreads = 256 + 128 * kDqSplit;  // warps 0-3 control, 4-7 epilogue, 8.. dequant
constexpr size_t kSmemBytes = 1024 + (size_t)kStages * (kXBytes + kWBytes) + 256;

static_assert(kAccCols + kStages * kACols <= kTmemCols, "TMEM budget");

// The work of one CTA as a sequence of segments (tile, k-blocks [kb0, kb1)).
// Tiles [0, t0) go whole, in rounds over the persistent grid: tiles
// blockIdx.x, blockIdx.x + gridDim.x, ... (t0 a multiple of the grid, so
// every CTA takes the same number of them, and the CTAs of a round work on
// neighbouring tiles, which share weight tiles and x in L2).  The remaining
// tiles [t0, tiles) -- the part of a last round that would leave SMs idle --
// are split evenly (stream-K): their k-blocks laid end to end as units
// u = (tile - t0) * kblocks + kb, CTA c taking [U c / G, U (c + 1) / G).
// A tile cut by a CTA boundary is computed in pieces whose fp32 sums go to a
// workspace and are added by streamk_fixup_kernel.  Only the first and last
// segments of a CTA's split range can be pieces.  t0 == tiles: no split.
struct Segments {
    int tiles, kblocks, t0;
    int tile;
    int64_t u, u1;
    __device__ Segments(int tiles_, int kblocks_, int t0_) : tiles(tiles_), kblocks(kblocks_), t0(t0_) {
        const int64_t units = (int64_t)(tiles - t0) * kblocks;
        tile = blockIdx.x;
        u = units * blockIdx.x / gridDim.x;
        u1 = units * (blockIdx.x + 1) / gridDim.x;
    }
    // `piece_index` counts the segments of the split range: 0 for the first.
    __device__ bool next(int &t, int &kb0, int &kb1, int &piece_index) {
        if (tile < t0) {
            t = tile, kb0 = 0, kb1 = kblocks, piece_index = -1;
            tile += gridDim.x;
            return true;
        }
        if (u >= u1) return false;
        t = t0 + (int)(u / kblocks);
        kb0 = (int)(u % kblocks);
        const int64_t left = u1 - u;
        kb1 = left < (int64_t)(kblocks - kb0) ? kb0 + (int)left : kblocks;
        piece_index = (tile == INT32_MAX) ? 1 : 0;
        tile = INT32_MAX;  // marks: the split range has started
        u += kb1 - kb0;
        return true;
    }
};

// Workspace slot of a piece: 2c for CTA c's first segment, 2c + 1 for its
// last.  A slot holds the piece's fp32 sums as [bx / 32][32][128]: chunk c
// of 32 batch rows, batch row j of the chunk, weight row r -- the epilogue's
// thread r writes v[j] at [c][j][r], so each warp store is 128 coalesced bytes.
__device__ __forceinline__ void store_piece(float *slot, int c, int r, const uint32_t (&v)[32]) {
    float *dst = slot + (size_t)c * 32 * 128 + r;
#pragma unroll
    for (int j = 0; j < 32; ++j) dst[j * 128] = __uint_as_float(v[j]);
}

// Adds the pieces of the split tiles, in k order, and writes them through
// the OutSpec.  `first.c[i]` is the first CTA boundary inside split tile i
// (the host lists them); blockIdx.x = i, and blockIdx.y picks the chunk
// [blockIdx.y * per, (blockIdx.y + 1) * per) of the tile's elements
// (gridDim.y chunks, sized so that the CTAs fill the GPU: a few split tiles
// can have ~100 pieces each).
constexpr int kMaxPiecesPerTile = 160;  // >= the grid (148 SMs) + 1

struct FixupList {
    int16_t c[kMaxPiecesPerTile];
};

__global__ void __launch_bounds__(256) streamk_fixup_kernel(const float *__restrict__ ws, OutSpec y, int m, int n,
                                                          int tiles_m, int bx, int kblocks, int t0, int64_t units,
                                                          int grid, FixupList first) {
    __shared__ const float *src[kMaxPiecesPerTile];
    __shared__ int npieces;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int c = first.c[blockIdx.x];
    auto u0 = [&](int cc) { return units * cc / grid; };
    const int64_t t = u0(c) / kblocks;                    // split tile t0 + t
    const size_t slot_floats = (size_t)bx * 128;
    if (threadIdx.x == 0) {
        // the CTAs holding the tile's pieces, in k order: c - 1 (the first), c, ...
        int np = 0;
        for (int cc = c - 1; cc < grid && (cc < c || u0(cc) < (t + 1) * kblocks) && np < kMaxPiecesPerTile; ++cc)
            src[np++] = ws + (2 * (size_t)cc + (u0(cc) >= t * kblocks ? 0 : 1)) * slot_floats;
        npieces = np;
    }
    __syncthreads();
    const int np = npieces;
    const int64_t tile = t0 + t;
    const int n0 = (int)(tile / tiles_m) * 128, m0 = (int)(tile % tiles_m) * bx;
    const int total = bx * 128, per = (total + (int)gridDim.y - 1) / (int)gridDim.y;
    const int e1 = min(total, (int)(blockIdx.y + 1) * per);
    for (int idx = (int)blockIdx.y * per + threadIdx.x; idx < e1; idx += blockDim.x) {
        const int r = idx & 127, bj = idx >> 7;           // bj = 32 chunk + j
        float v = src[0][idx];
        // eight loads in flight, then the adds in k order
        for (int i0 = 1; i0 < np; i0 += 8) {
            float part[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) part[i] = i0 + i < np ? src[i0 + i][idx] : 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (i0 + i < np) v += part[i];
        }
        const int b = m0 + bj, f = n0 + r;
        if (b < m && f < n) y.store(b, f, v);
    }
}

// SiLU-gate tiles (gate_n > 0): the weights are an MLP's [gate; up] stack
// of n = 2 gate_n rows and the output y = silu(x . Wg^T) * (x . Wu^T) has
// gate_n features.  A 128-row tile then holds 64 features: in TMEM lane
// quarter q, lanes 0-15 are the gate rows of features f0 + 16 q + (0..15) and
// lanes 16-31 the up rows of the same features, so the epilogue pairs them
// with one shuffle.  f0 = 64 (tile / tiles_m) = n0 / 2.  Gate rows past gate_n
// read up rows and up rows past n read zeros (TMA fill); neither is stored.
__device__ __forceinline__ int tile_weight_row(int gate_n, int n0, int r) {
    if (gate_n == 0) return n0 + r;
    const int q = r >> 5, l = r & 31;
    return ((l & 16) ? gate_n : 0) + (n0 >> 1) + 16 * q + (l & 15);
}

// The packed tile of one k-block: one 128-row TMA box, or in SiLU-gate mode
// eight 16-row boxes (smem rows 16 b ..: gate rows for even b, up rows for
// odd b, of lane quarter b / 2) -- the same 4 KB either way.
__device__ __forceinline__ void load_weight_tile(uint8_t *dst, const CUtensorMap *wmap, uint64_t *bar, int kb,
                                                 int n0, int gate_n) {
    if (gate_n == 0) {
        tma_load_2d(dst, wmap, bar, kb * (kBK / 2), n0);
        return;
    }
#pragma unroll
    for (int b = 0; b < 8; ++b)
        tma_load_2d(dst + b * 16 * (kBK / 2), wmap, bar, kb * (kBK / 2),
                    ((b & 1) ? gate_n : 0) + (n0 >> 1) + 16 * (b >> 1));
}

// Epilogue of a run of 32 batch rows of one TMEM lane: y.store_run, or in
// SiLU-gate mode silu(gate) * up.  There lane l < 16 holds the gate sums of
// feature l and lane l + 16 the up sums: the partners swap their values, lane
// l computes batch rows 0-15 of feature l and lane l + 16 rows 16-31, so all
// 32 lanes share the work.  silu(g) = g / (1 + e^-g) with the fast exp and
// division intrinsics (a few ulp): the epilogue holds the tile's TMEM
// accumulator until it is done, so its cost is on the GEMM's critical path.
template <int CNT>
__device__ __forceinline__ void store_tile_run(const OutSpec &y, int64_t b0, int64_t bend, int n, int gate_n, int n0,
                                               int q, int lane, uint32_t (&v)[CNT]) {
    static_assert(CNT == 32, "one TMEM load of 32 batch rows");
    if (gate_n == 0) {
        const int row = n0 + q * 32 + lane;
        if (row < n) y.store_run(b0, bend, row, v);
        return;
    }
    const bool lo = lane < 16;
    uint32_t o[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        // partner values of rows j and j + 16 (xor 16: gate <-> up lane)
        const float pa = __shfl_xor_sync(0xffffffffu, __uint_as_float(v[j]), 16);
        const float pb = __shfl_xor_sync(0xffffffffu, __uint_as_float(v[j + 16]), 16);
        const float g = lo ? __uint_as_float(v[j]) : pb;
        const float u = lo ? pa : __uint_as_float(v[j + 16]);
        o[j] = __float_as_uint(__fdividef(g, 1.0f + __expf(-g)) * u);
    }
    const int f = (n0 >> 1) + 16 * q + (lane & 15);
    if (f < gate_n) y.store_run(b0 + (lo ? 0 : 16), bend, f, o);
}

template <typename XT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_int4_tcgen05_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                             const float *__restrict__ scales, OutSpec y, int m, int n, int kp, int g, int t0,
                             float *__restrict__ ws, int gate_n) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    uint8_t *xbuf = smem;                                    // [S][256 rows][128 B], swizzled
    uint8_t *wbuf = xbuf + (size_t)kStages * kXBytes;        // [S][128 rows][32 B]
    uint64_t *full = reinterpret_cast<uint64_t *>(wbuf + (size_t)kStages * kWBytes);
    uint64_t *deq = full + kStages;
    uint64_t *empty = deq + kStages;
    uint64_t *acc_full = empty + kStages;
    uint64_t *acc_empty = acc_full + 1;
    uint64_t *mma_done = acc_empty + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma_done + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles_n = (n + kBN - 1) / kBN, tiles_m = (m + kBX - 1) / kBX;
    const int tiles = tiles_n * tiles_m;
    const int kblocks = (kp + kBK - 1) / kBK;
    const int groups = kp / g;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);   // producer's expect_tx arrival
            mbar_init(&deq[s], 4 * kDqSplit);  // one arrival per dequant warp
            mbar_init(&empty[s], 1);  // tcgen05.commit
        }
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, 4);
        mbar_init(mma_done, 1);
        fence_barrier_init();
    }
    if (warp == 2) {
        tmem_alloc(tmem_slot, kTmemCols);
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
            Segments seg(tiles, kblocks, t0);
            int tile, kb0, kb1, pi;
            while (ok && seg.next(tile, kb0, kb1, pi)) {
                const int n0 = (tile / tiles_m) * kBN, m0 = (tile % tiles_m) * kBX;
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const int s = it % kStages, r = it / kStages;
                    if (r > 0 && !(ok = mbar_wait(&empty[s], (r - 1) & 1))) break;
                    mbar_arrive_expect_tx(&full[s], kXBytes + kWBytes);
                    tma_load_2d(xbuf + (size_t)s * kXBytes, &xmap, &full[s], kb * kBK, m0);
                    load_weight_tile(wbuf + (size_t)s * kWBytes, &wmap, &full[s], kb, n0, gate_n);
                }
            }
            // Drain: every issued stage's copies must land before the CTA
            // exits (normally the consumers have waited for all of them).
            for (int j = (it > kStages ? it - kStages : 0); j < it; ++j)
                mbar_wait(&full[j % kStages], (j / kStages) & 1);
        }
    } else if (warp == 1) {
        // ----------------------------------------------------------- MMA
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_f16(kBN, kBX, std::is_same<XT, __nv_bfloat16>::value);
            int it = 0, ti = 0;
            bool ok = true;
            Segments seg(tiles, kblocks, t0);
            int tile, kb0, kb1, pi;
            for (; ok && seg.next(tile, kb0, kb1, pi); ++ti) {
                if (ti > 0 && !(ok = mbar_wait(acc_empty, (ti - 1) & 1))) break;
                tc_fence_after();
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const int s = it % kStages, r = it / kStages;
                    if (!(ok = mbar_wait(&full[s], r & 1))) break;
                    if (!(ok = mbar_wait(&deq[s], r & 1))) break;
                    tc_fence_after();
                    const uint64_t bdesc = umma_desc_sw128(smem_u32(xbuf + (size_t)s * kXBytes));
                    const uint32_t a_tmem = tmem + kAccCols + s * kACols;
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk)
                        tc_mma_ts(tmem, a_tmem + kk * 8, bdesc + (uint64_t)(kk * 32 / 16), idesc,
                                  (kb != kb0 || kk != 0) ? 1u : 0u);
                    tc_commit(&empty[s]);
                }
                if (ok) tc_commit(acc_full);
            }
            // Every MMA this thread issued has completed once mma_done fires.
            tc_commit(mma_done);
            mbar_wait(mma_done, 0);
        }
    } else if (warp >= 8) {
        // ------------------------------------------------------- dequant
        const int d = warp - 8;
        const int q = d & 3;            // TMEM lane quarter (= warp % 4)
        const int part = d >> 2;        // which kDqWords words of the row's k-block
        const int r = q * 32 + lane;    // weight row within the tile
        int it = 0;
        bool ok = true;
        Segments seg(tiles, kblocks, t0);
        int tile, kb0, kb1, pi;
        while (ok && seg.next(tile, kb0, kb1, pi)) {
            const int n0 = (tile / tiles_m) * kBN;
            const float *srow = scales + (size_t)min(tile_weight_row(gate_n, n0, r), n - 1) * groups;
            for (int kb = kb0; kb < kb1; ++kb, ++it) {
                const int s = it % kStages, rd = it / kStages;
                const int c0 = kb * kBK;
                // words 0-3 of a row's k-block are columns c0..c0+31 (scale
                // s0), words 4-7 the next 32 (s1)
                const float s0 = __ldg(srow + min(c0 / g, groups - 1));
                const float s1 = kDqSplit == 1 || part * kDqWords >= 4 ? __ldg(srow + min((c0 + 32) / g, groups - 1))
                                                                      : s0;
                // Warp-uniform outcome: tcgen05.st below is .sync.aligned.
                ok = __all_sync(0xffffffffu, mbar_wait(&full[s], rd & 1));
                if (!ok) break;
                uint32_t words[kDqWords];
                const uint8_t *src = wbuf + (size_t)s * kWBytes + r * 32 + part * kDqWords * 4;
                if constexpr (kDqWords % 4 == 0) {
#pragma unroll
                    for (int v = 0; v < kDqWords; v += 4) {
                        const uint4 wv = *reinterpret_cast<const uint4 *>(src + 4 * v);
                        words[v] = wv.x, words[v + 1] = wv.y, words[v + 2] = wv.z, words[v + 3] = wv.w;
                    }
                } else {
                    const uint2 wv = *reinterpret_cast<const uint2 *>(src);
                    words[0] = wv.x, words[1] = wv.y;
                }
                const DqScale d0 = make_dq_scale(s0), d1 = make_dq_scale(s1);
                uint32_t a[4 * kDqWords];
                auto run = [&](auto fast_tag) {
                    constexpr bool FAST = decltype(fast_tag)::value;
#pragma unroll
                    for (int wd = 0; wd < kDqWords; ++wd) {
                        const DqScale &ds = part * kDqWords + wd < 4 ? d0 : d1;
                        uint32_t h0[2], h1[2];
                        dq_half<XT, 0, FAST>(words[wd], ds, h0);
                        dq_half<XT, 1, FAST>(words[wd], ds, h1);
                        a[4 * wd + 0] = h0[0];
                        a[4 * wd + 1] = h0[1];
                        a[4 * wd + 2] = h1[0];
                        a[4 * wd + 3] = h1[1];
                    }
                };
                if (__all_sync(0xffffffffu, d0.fast && d1.fast))
                    run(std::true_type{});
                else
                    run(std::false_type{});
                tmem_st_32x32b<4 * kDqWords>(
                    tmem + ((uint32_t)(q * 32) << 16) + kAccCols + s * kACols + part * 4 * kDqWords, a);
                tc_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&deq[s]);
            }
        }
    } else if (warp >= 4) {
        // ------------------------------------------------------ epilogue
        const int q = warp - 4;
        int ti = 0;
        bool ok = true;
        Segments seg(tiles, kblocks, t0);
        int tile, kb0, kb1, pi;
        for (; ok && seg.next(tile, kb0, kb1, pi); ++ti) {
            const int n0 = (tile / tiles_m) * kBN, m0 = (tile % tiles_m) * kBX;
            ok = __all_sync(0xffffffffu, mbar_wait(acc_full, ti & 1));  // tcgen05.ld is .sync.aligned
            if (!ok) break;
            tc_fence_after();
            const bool piece = kb0 != 0 || kb1 != kblocks;  // (never in SiLU-gate mode)
            float *slot = ws + (2 * (size_t)blockIdx.x + (pi == 0 ? 0 : 1)) * (size_t)(kAccCols * kBN);
#pragma unroll 1
            for (int c = 0; c < kAccCols / 32; ++c) {
                uint32_t v[32];
                tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + c * 32, v);
                tc_wait_ld();
                if (piece)
                    store_piece(slot, c, q * 32 + lane, v);
                else
                    store_tile_run(y, m0 + c * 32, m, n, gate_n, n0, q, lane, v);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty);
        }
    }

    // Lane 0 of warps 0 and 1 ran their roles alone: converge each warp
    // before the CTA-wide barrier (an aligned barrier in a diverged warp is
    // undefined), so that TMEM is released only after every role is done.
    __syncwarp();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// ---------------------------------------------------------- wide tiles --
//
// For M >= 1024: the same roles, but each dequantized A slot feeds two MMAs,
// one per half of a batch tile of 2 * NB rows (NB <= 224, a multiple of 16),
// into two accumulators -- half the weight dequantizations per flop of the
// 256-row tiles above, which the exact rounding makes the costly part.
// TMEM: accumulators in columns [0, 2 NB), two A slots of 32 columns at 448.
// Shared memory: 3 stages of (2 NB x 128 B of x, loaded as two NB-row TMA
// boxes, + the 4 KB packed tile).  The A-slot ring (2) is decoupled from the
// stage ring (3): deq[a] publishes a written slot, a_empty[a] (tcgen05.commit)
// frees it for the dequant warps.
constexpr int kWideStages = 3;
constexpr int kWideMaxNB = 224;
constexpr int kWideXBytes = 2 * kWideMaxNB * kBK * 2;  // 56 KB x tile per stage
constexpr int kWideACol = 448;                           // first A-slot column
constexpr size_t kWideSmemBytes = 1024 + (size_t)kWideStages * (kWideXBytes + kWBytes) + 256;

static_assert(kWideACol + 2 * kACols <= kTmemCols, "wide TMEM budget");

template <typename XT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_int4_tcgen05_wide_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                                  const float *__restrict__ scales, OutSpec y, int m, int n, int kp, int g, int nb,
                                  int t0, float *__restrict__ ws, int gate_n) {
    static_assert(kDqSplit == 1, "the wide kernel keeps one dequant warp per TMEM lane quarter");
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    uint8_t *xbuf = smem;                                        // [S][2 nb rows][128 B], swizzled
    uint8_t *wbuf = xbuf + (size_t)kWideStages * kWideXBytes;    // [S][128 rows][32 B]
    uint64_t *full = reinterpret_cast<uint64_t *>(wbuf + (size_t)kWideStages * kWBytes);
    uint64_t *empty = full + kWideStages;
    uint64_t *deq = empty + kWideStages;  // [2] A slots
    uint64_t *a_empty = deq + 2;          // [2]
    uint64_t *acc_full = a_empty + 2;
    uint64_t *acc_empty = acc_full + 1;
    uint64_t *mma_done = acc_empty + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma_done + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int bx = 2 * nb;  // batch rows per tile
    const int tiles_n = (n + kBN - 1) / kBN, tiles_m = (m + bx - 1) / bx;
    const int tiles = tiles_n * tiles_m;
    const int kblocks = (kp + kBK - 1) / kBK;
    const int groups = kp / g;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kWideStages; ++s) {
            mbar_init(&full[s], 1);   // producer's expect_tx arrival
            mbar_init(&empty[s], 1);  // tcgen05.commit
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&deq[a], 4);      // one arrival per dequant warp
            mbar_init(&a_empty[a], 1);  // tcgen05.commit
        }
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, 4);
        mbar_init(mma_done, 1);
        fence_barrier_init();
    }
    if (warp == 2) {
        tmem_alloc(tmem_slot, kTmemCols);
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
            const uint32_t tx = (uint32_t)(bx * kBK * 2 + kWBytes);
            Segments seg(tiles, kblocks, t0);
            int tile, kb0, kb1, pi;
            while (ok && seg.next(tile, kb0, kb1, pi)) {
                const int n0 = (tile / tiles_m) * kBN, m0 = (tile % tiles_m) * bx;
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const int s = it % kWideStages, r = it / kWideStages;
                    if (r > 0 && !(ok = mbar_wait(&empty[s], (r - 1) & 1))) break;
                    uint8_t *xs = xbuf + (size_t)s * kWideXBytes;
                    mbar_arrive_expect_tx(&full[s], tx);
                    tma_load_2d(xs, &xmap, &full[s], kb * kBK, m0);
                    tma_load_2d(xs + nb * 128, &xmap, &full[s], kb * kBK, m0 + nb);
                    load_weight_tile(wbuf + (size_t)s * kWBytes, &wmap, &full[s], kb, n0, gate_n);
                }
            }
            // Drain: every issued stage's copies land before the CTA exits.
            for (int j = (it > kWideStages ? it - kWideStages : 0); j < it; ++j)
                mbar_wait(&full[j % kWideStages], (j / kWideStages) & 1);
        }
    } else if (warp == 1) {
        // ----------------------------------------------------------- MMA
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_f16(kBN, nb, std::is_same<XT, __nv_bfloat16>::value);
            int it = 0, ti = 0;
            bool ok = true;
            Segments seg(tiles, kblocks, t0);
            int tile, kb0, kb1, pi;
            for (; ok && seg.next(tile, kb0, kb1, pi); ++ti) {
                if (ti > 0 && !(ok = mbar_wait(acc_empty, (ti - 1) & 1))) break;
                tc_fence_after();
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const int s = it % kWideStages, a = it & 1;
                    if (!(ok = mbar_wait(&full[s], (it / kWideStages) & 1))) break;
                    if (!(ok = mbar_wait(&deq[a], (it >> 1) & 1))) break;
                    tc_fence_after();
                    const uint32_t xaddr = smem_u32(xbuf + (size_t)s * kWideXBytes);
                    const uint64_t b0 = umma_desc_sw128(xaddr), b1 = umma_desc_sw128(xaddr + nb * 128);
                    const uint32_t a_tmem = tmem + kWideACol + a * kACols;
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk) {
                        const uint32_t acc = (kb != kb0 || kk != 0) ? 1u : 0u;
                        tc_mma_ts(tmem, a_tmem + kk * 8, b0 + (uint64_t)(kk * 32 / 16), idesc, acc);
                        tc_mma_ts(tmem + nb, a_tmem + kk * 8, b1 + (uint64_t)(kk * 32 / 16), idesc, acc);
                    }
                    tc_commit(&empty[s]);
                    tc_commit(&a_empty[a]);
                }
                if (ok) tc_commit(acc_full);
            }
            // Every MMA this thread issued has completed once mma_done fires.
            tc_commit(mma_done);
            mbar_wait(mma_done, 0);
        }
    } else if (warp >= 8) {
        // ------------------------------------------------------- dequant
        const int q = warp - 8;         // TMEM lane quarter
        const int r = q * 32 + lane;    // weight row within the tile
        int it = 0;
        bool ok = true;
        Segments seg(tiles, kblocks, t0);
        int tile, kb0, kb1, pi;
        while (ok && seg.next(tile, kb0, kb1, pi)) {
            const int n0 = (tile / tiles_m) * kBN;
            const float *srow = scales + (size_t)min(tile_weight_row(gate_n, n0, r), n - 1) * groups;
            for (int kb = kb0; kb < kb1; ++kb, ++it) {
                const int s = it % kWideStages, a = it & 1;
                const int c0 = kb * kBK;
                const float s0 = __ldg(srow + min(c0 / g, groups - 1));
                const float s1 = __ldg(srow + min((c0 + 32) / g, groups - 1));
                // Warp-uniform outcomes: tcgen05.st below is .sync.aligned.
                ok = __all_sync(0xffffffffu, mbar_wait(&full[s], (it / kWideStages) & 1));
                if (ok && it >= 2) ok = __all_sync(0xffffffffu, mbar_wait(&a_empty[a], ((it >> 1) - 1) & 1));
                if (!ok) break;
                const uint4 w0 = *reinterpret_cast<const uint4 *>(wbuf + (size_t)s * kWBytes + r * 32);
                const uint4 w1 = *reinterpret_cast<const uint4 *>(wbuf + (size_t)s * kWBytes + r * 32 + 16);
                const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
                const DqScale d0 = make_dq_scale(s0), d1 = make_dq_scale(s1);
                uint32_t av[32];
                auto run = [&](auto fast_tag) {
                    constexpr bool FAST = decltype(fast_tag)::value;
#pragma unroll
                    for (int wd = 0; wd < 8; ++wd) {
                        uint32_t h0[2], h1[2];
                        dq_half<XT, 0, FAST>(words[wd], wd < 4 ? d0 : d1, h0);
                        dq_half<XT, 1, FAST>(words[wd], wd < 4 ? d0 : d1, h1);
                        av[4 * wd + 0] = h0[0];
                        av[4 * wd + 1] = h0[1];
                        av[4 * wd + 2] = h1[0];
                        av[4 * wd + 3] = h1[1];
                    }
                };
                if (__all_sync(0xffffffffu, d0.fast && d1.fast))
                    run(std::true_type{});
                else
                    run(std::false_type{});
                tmem_st_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + kWideACol + a * kACols, av);
                tc_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&deq[a]);
            }
        }
    } else if (warp >= 4) {
        // ------------------------------------------------------ epilogue
        const int q = warp - 4;
        int ti = 0;
        bool ok = true;
        Segments seg(tiles, kblocks, t0);
        int tile, kb0, kb1, pi;
        for (; ok && seg.next(tile, kb0, kb1, pi); ++ti) {
            const int n0 = (tile / tiles_m) * kBN, m0 = (tile % tiles_m) * bx;
            ok = __all_sync(0xffffffffu, mbar_wait(acc_full, ti & 1));  // tcgen05.ld is .sync.aligned
            if (!ok) break;
            tc_fence_after();
            const bool piece = kb0 != 0 || kb1 != kblocks;  // (never in SiLU-gate mode)
            float *slot = ws + (2 * (size_t)blockIdx.x + (pi == 0 ? 0 : 1)) * (size_t)(bx * kBN);
#pragma unroll 1
            for (int c = 0; c < bx / 32; ++c) {
                uint32_t v[32];
                tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + c * 32, v);
                tc_wait_ld();
                if (piece)
                    store_piece(slot, c, q * 32 + lane, v);
                else
                    store_tile_run(y, m0 + c * 32, m, n, gate_n, n0, q, lane, v);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty);
        }
    }

    // Lane 0 of warps 0 and 1 ran their roles alone: converge each warp
    // before the CTA-wide barrier (an aligned barrier in a diverged warp is
    // undefined), so that TMEM is released only after every role is done.
    __syncwarp();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

int allow_smem(const void *kern, size_t bytes) {
    static std::mutex mu;
    static std::set<std::pair<const void *, int>> done;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    if (done.count({kern, dev})) return OQ_OK;
    OQ_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    done.insert({kern, dev});
    return OQ_OK;
}

// Batch rows from which the wide-tile kernel is considered: below it the
// 256-row tiles waste less on the ragged last tile than the wide ones save.
constexpr int64_t kWideMinM = 1024;

// NB of the wide tiles for M: the fewest tiles of at most 2 x 224 rows, then
// the smallest NB (a multiple of 16) whose tiles cover M.
inline int wide_nb(int64_t m) {
    const int64_t tiles_m = cdiv(m, 2 * kWideMaxNB);
    return (int)std::min<int64_t>(kWideMaxNB, cdiv(cdiv(cdiv(m, tiles_m), 2), 16) * 16);
}

// The launch plan: 256-row or wide tiles, and whether the tiles of the last
// round are split (stream-K).  A wave model of the persistent grid picks it:
// each tile costs its batch rows plus the dequant of its weight tile (about
// 128 rows' worth, measured); whole tiles go in rounds over the SMs, the last
// round often part-empty (148 SMs divide few tile counts); the split spreads
// that last round's tiles evenly over all SMs.  Measured on the Llama-3-70B
// MLP shapes, the split costs about a quarter round more than that (the
// pieces' epilogues, the fix-up launch, and x streamed out of step with the
// other SMs), and it only pays when the last round would be less than ~45 %
// full: from 0.89 to 1.03 PFLOP/s (gate/up at M = 512, 4 of 448 tiles left
// over), 0.92 -> 1.23 (down, M = 2048), 1.07 -> 1.17 (down, M = 8192); with
// 57-86 % full last rounds it lost 0-9 %.  The split needs a caller
// workspace of ws_bytes.
struct GemmPlan {
    bool wide = false, split = false;
    int nb = 0, bx = kBX;
    int64_t tiles = 0, grid = 0, kblocks = 0, t0 = 0;  // t0: first split tile (tiles: none)
    size_t ws_bytes = 0;
};

inline GemmPlan plan_gemm(int64_t m, int64_t n, int64_t k, int g, bool allow_split) {
    constexpr int64_t kDequantRows = 128;
    constexpr double kSplitOverhead = 0.25;  // rounds
    constexpr double kSplitMaxLastRound = 0.45;
    const int64_t sms = sm_count(), tiles_n = cdiv(n, kBN);
    const int64_t kblocks = cdiv(cdiv(k, g) * g, kBK);
    GemmPlan best;
    double best_cost = 0.0;
    auto consider = [&](bool wide, int nb, int bx, bool split) {
        const int64_t tiles = tiles_n * cdiv(m, bx);
        const double per_tile = (double)(bx + kDequantRows);
        int64_t grid = std::min<int64_t>(tiles, sms), t0 = tiles;
        double cost = per_tile * (double)cdiv(tiles, sms);
        if (split) {
            t0 = tiles / sms * sms;  // whole rounds first
            const int64_t rest = tiles - t0;
            grid = std::min<int64_t>(std::min<int64_t>(sms, kMaxPiecesPerTile - 1), rest * kblocks + t0);
            if (rest == 0 || rest * kblocks < grid) return;  // nothing to split, or pieces under a k-block
            if ((double)rest / (double)sms > kSplitMaxLastRound) return;
            cost = per_tile * ((double)(t0 / sms) + (double)rest / (double)sms + kSplitOverhead);
        }
        if (best.tiles != 0 && cost >= best_cost) return;
        best_cost = cost;
        best.wide = wide, best.split = split, best.nb = nb, best.bx = bx, best.tiles = tiles, best.kblocks = kblocks;
        best.grid = grid, best.t0 = t0;
        best.ws_bytes = split ? (size_t)2 * grid * bx * kBN * sizeof(float) : 0;
    };
    consider(false, 0, kBX, false);
    if (m >= kWideMinM) consider(true, wide_nb(m), 2 * wide_nb(m), false);
    if (allow_split) {
        consider(false, 0, kBX, true);
        if (m >= kWideMinM) consider(true, wide_nb(m), 2 * wide_nb(m), true);
    }
    return best;
}

// n: weight rows (2 gate_n in SiLU-gate mode, which never splits).
template <typename XT>
int launch(const XT *x, CUtensorMapDataType xtype, const uint8_t *packed, const float *scales, OutSpec y, int64_t m,
           int64_t n, int64_t k, int g, void *ws, size_t ws_bytes, int64_t gate_n, cudaStream_t st) {
    GemmPlan plan = plan_gemm(m, n, k, g, ws != nullptr && gate_n == 0);
    if (plan.split && ws_bytes < plan.ws_bytes) plan = plan_gemm(m, n, k, g, false);
    const int64_t kp = cdiv(k, g) * g;
    CUtensorMap xmap, wmap;
    int rc = make_tensor_map_2d(&xmap, x, xtype, 2, (uint64_t)k, (uint64_t)m, (uint64_t)(k * 2), kBK,
                                (uint32_t)(plan.wide ? plan.nb : kBX), CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != OQ_OK) return rc;
    rc = make_tensor_map_2d(&wmap, packed, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)(kp / 2), (uint64_t)n,
                            (uint64_t)(kp / 2), kBK / 2, gate_n ? 16 : kBN, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc != OQ_OK) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)plan.grid);
    cfg.blockDim = dim3(kThreads);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    float *wsf = static_cast<float *>(ws);
    cudaError_t err;
    if (plan.wide) {
        auto kern = gemm_int4_tcgen05_wide_kernel<XT>;
        rc = allow_smem(reinterpret_cast<const void *>(kern), kWideSmemBytes);
        if (rc != OQ_OK) return rc;
        cfg.dynamicSmemBytes = kWideSmemBytes;
        err = cudaLaunchKernelEx(&cfg, kern, xmap, wmap, scales, y, (int)m, (int)n, (int)kp, g, plan.nb, (int)plan.t0,
                                 wsf, (int)gate_n);
    } else {
        auto kern = gemm_int4_tcgen05_kernel<XT>;
        rc = allow_smem(reinterpret_cast<const void *>(kern), kSmemBytes);
        if (rc != OQ_OK) return rc;
        cfg.dynamicSmemBytes = kSmemBytes;
        err = cudaLaunchKernelEx(&cfg, kern, xmap, wmap, scales, y, (int)m, (int)n, (int)kp, g, (int)plan.t0, wsf,
                                 (int)gate_n);
    }
    if (err != cudaSuccess) {
        set_error("int4_linear (tcgen05 GEMM): launch failed: %s", cudaGetErrorString(err));
        return OQ_ERR_CUDA;
    }
    if (!plan.split || plan.grid < 2) return OQ_OK;
    // The split tiles, each by the first CTA boundary inside it.
    const int64_t split_units = (plan.tiles - plan.t0) * plan.kblocks;
    FixupList first = {};
    int split_tiles = 0;
    int64_t last = -1;
    for (int64_t c = 1; c < plan.grid; ++c) {
        const int64_t ub = split_units * c / plan.grid;
        if (ub % plan.kblocks != 0 && ub / plan.kblocks != last) {
            first.c[split_tiles++] = (int16_t)c;
            last = ub / plan.kblocks;
        }
    }
    if (split_tiles == 0) return OQ_OK;
    // Chunks per split tile: about four CTAs per SM over all split tiles.
    const int64_t chunks = std::min<int64_t>(256, std::max<int64_t>(4, cdiv(4 * sm_count(), split_tiles)));
    cudaLaunchConfig_t fcfg = cfg;
    fcfg.gridDim = dim3((unsigned)split_tiles, (unsigned)chunks);
    fcfg.blockDim = dim3(256);
    fcfg.dynamicSmemBytes = 0;
    err = cudaLaunchKernelEx(&fcfg, streamk_fixup_kernel, (const float *)wsf, y, (int)m, (int)n,
                             (int)cdiv(m, plan.bx), plan.bx, (int)plan.kblocks, (int)plan.t0, split_units,
                             (int)plan.grid, first);
    if (err != cudaSuccess) {
        set_error("int4_linear (tcgen05 GEMM fix-up): launch failed: %s", cudaGetErrorString(err));
        return OQ_ERR_CUDA;
    }
    return OQ_OK;
}

}  // namespace

// The tcgen05 GEMM takes: K % 8 == 0 (16-byte x rows for TMA), a group size
// that is a multiple of 32 (each 32-column half of a k-block has one scale)
// with KP % 32 == 0, 16-byte aligned x and packed, and sizes below 2^31.
int gemm_tcgen05_supported(int64_t m, int64_t n, int64_t k, int g, const void *x, const uint8_t *packed,
                           const float *y) {
    (void)y;
    if (m < 1 || n < 1 || k < 1 || g < 32 || g % 32 != 0) return 0;
    const int64_t kp = cdiv(k, g) * g;
    if (k % 8 != 0 || kp % 32 != 0) return 0;
    if (!aligned(x, 16) || !aligned(packed, 16)) return 0;
    if (m >= (1ll << 31) || n >= (1ll << 31) || kp >= (1ll << 31) || m * n >= (1ll << 40)) return 0;
    return 1;
}

int gemm_tcgen05_launch(const void *x, int x_dtype, const uint8_t *packed, const float *scales, OutSpec y, int64_t m,
                        int64_t n, int64_t k, int g, void *ws, size_t ws_bytes, cudaStream_t st, int64_t gate_n) {
    // gate_n > 0: SiLU-gate mode -- `packed` / `scales` hold the [gate; up]
    // stack of n = 2 gate_n rows and y gets gate_n features (no workspace).
    if (x_dtype == OQ_BF16)
        return launch(static_cast<const __nv_bfloat16 *>(x), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, packed, scales, y, m,
                      n, k, g, ws, ws_bytes, gate_n, st);
    return launch(static_cast<const __half *>(x), CU_TENSOR_MAP_DATA_TYPE_FLOAT16, packed, scales, y, m, n, k, g, ws,
                  ws_bytes, gate_n, st);
}

size_t gemm_tcgen05_workspace_bytes(int64_t m, int64_t n, int64_t k, int g) {
    return plan_gemm(m, n, k, g, true).ws_bytes;
}

}  // namespace oq
