// linear.cu -- the weight contractions either side of the hot path on the
// sm_100a tensor cores, with the path's own epilogues fused:
//   y = act(x . w^T + bias) + resid
// replacing the GEMVs computeQKVKernel, projectionKernel, ffnUpKernel and
// ffnDownKernel (transformer.cu:187-294).  The reference computes these in
// fp32 on the CUDA cores; here every operand arrives as a tf32 pair
// (hi, lo) and the tensor cores form hi.hi + hi.lo + lo.hi.
//
// Accuracy.  The pair products are within ~2^-22 of the fp32 products, but
// the tensor core's f32 accumulator loses low-order bits on every addition
// (measured on B200, RMS error over sum |x w|: with the whole K sum in TMEM
// 3e-7 at K = 768 to 9e-7 at K = 6400, 10-30x an fp32 SGEMM's 2.8e-8, and
// growing with K).  So TMEM only ever holds the partial sum of one K chunk
// of kLinChunkK, and the epilogue warps add each chunk into fp32 registers
// (round to nearest).  At 128 the RMS error is 5.5e-8 / 2.8e-8 / 1.9e-8 at
// K = 768 / 3072 / 6400, fp32-grade; 64 halves it and costs 5% more time,
// 256 doubles it and saves 5%.
//
// Kernel layout (one CTA per SM, persistent over 128 x 256 output tiles):
//   warp 0      TMA producer: per K block, the x_hi, x_lo, w_hi, w_lo tiles
//               (K-major, 64- or 128-byte swizzled rows) into a ring of
//               shared-memory stages, completion counted on full[stage]
//   warp 1      owns the 512 TMEM columns (two 128 x 256 f32 chunk
//               buffers); one thread issues tcgen05.mma (kind::tf32, M 128,
//               N 256, K 8) per product term and K step; tcgen05.commit
//               frees a stage (empty[stage]) or hands a finished chunk to the
//               epilogue (chunk_full[buffer])
//   warps 2-9   epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31 (one
//               output row per thread) and columns 128 ((w - 2) / 4) .. +127;
//               per chunk, tcgen05.ld and add into 128 fp32 registers, then
//               chunk_empty lets the MMA thread refill the buffer (so the
//               next chunk's MMAs overlap this chunk's read-out); per tile,
//               + bias, GELU, + resid, optional tf32 split, 16-byte stores
// Every mbarrier wait is bounded (1 s, %globaltimer): a wait that runs out
// sets the CTA's abort word, every role leaves its loop, the producer waits
// (bounded) for its loads in flight, the MMA thread for its MMAs, TMEM is
// freed, and GBX_LINEAR_TIMEOUT is OR-ed into err_flag.  No cluster
// multicast: every TMA load fills this CTA's own shared memory.
#include <atomic>
#include <cuda.h>
#include <stdlib.h>

#include <mutex>

#include "gbx_common.cuh"
#include "gelu.cuh"
#include "tcgen05.cuh"
#include "tensormap.cuh"
#include "tf32.cuh"

namespace gbx {

constexpr int kLinBM = 128;           // tile rows = TMEM lanes
constexpr int kLinBN = 256;           // tile columns = TMEM columns of one chunk buffer
constexpr int kLinEpiWarps = 8;       // two per TMEM lane quarter, 128 columns each
constexpr int kLinEpiThreads = 32 * kLinEpiWarps;
constexpr int kLinThreads = 64 + kLinEpiThreads;
constexpr int kLinEpiCols = kLinBN / 2;
constexpr int kLinBuffers = 2;        // 2 x 256 = all 512 TMEM columns
constexpr int kLinTmemCols = kLinBuffers * kLinBN;
#ifndef GBX_LINEAR_CHUNK_K
#define GBX_LINEAR_CHUNK_K 128
#endif
constexpr int kLinChunkK = GBX_LINEAR_CHUNK_K;   // K elements summed in TMEM before each fp32 promotion
constexpr uint64_t kLinWaitNs = kDeviceWaitNs;
// Heads mode: per epilogue warp, a 32-row x 16-column staging block in
// shared memory (after the barriers) for coalesced output stores.
constexpr int kLinStageFloats = 32 * 16;
constexpr size_t kLinEpiStageBytes = (size_t)kLinEpiWarps * kLinStageFloats * sizeof(float) + 16;

// Shared-memory ring and barrier layout.  PAIR: a cluster of two CTAs runs
// one M 256 x N 256 MMA (cta_group::2); each CTA holds its 128 x rows and
// half (128) of the w rows, so a stage is 4 tiles of 128 rows.
template <int BK, bool PAIR>
struct LinCfg {
    static constexpr int row_bytes = BK * 4;             // 64 or 128: the swizzle width
    static constexpr int a_rows = kLinBM;                 // x rows in this CTA
    static constexpr int b_rows = PAIR ? kLinBN / 2 : kLinBN;   // w rows in this CTA
    static constexpr int a_bytes = a_rows * row_bytes;   // one x tile
    static constexpr int b_bytes = b_rows * row_bytes;   // one w tile
    static constexpr int stage_bytes = 2 * a_bytes + 2 * b_bytes;
    static constexpr int stages = (196 * 1024) / stage_bytes;   // BK 16: 4 (6 paired), BK 32: 2 (3 paired)
    static constexpr int ksteps = BK / 8;                       // tf32 MMA K = 8 (32 bytes)
    static constexpr int chunk_blocks = kLinChunkK / BK;          // K blocks per chunk
    static constexpr int tile_rows = PAIR ? 2 * kLinBM : kLinBM;  // output rows per tile
    static constexpr int nbars = 2 * stages + 3 * kLinBuffers + 1;
    static constexpr size_t smem = (size_t)stages * stage_bytes + 1024 + 8 * nbars + 16;
    static_assert(kLinChunkK % 32 == 0, "a chunk is whole K blocks");
    static_assert(BK == 16 || BK == 32, "swizzle width");
    static_assert(stages >= 2, "pipeline depth");
    static_assert(a_bytes % 1024 == 0 && b_bytes % 1024 == 0, "tiles stay aligned to the swizzle repeat");
};

struct LinearArgs {
    const float* bias;
    const float* resid;
    float* y;
    float* y_lo;
    int* err;
    int64_t M;
    int N;
    int K;
    int m_blocks;
    int n_blocks;
    int k_blocks;
    int tiles;
    int act;
    int has_xlo;
    int has_wlo;
    // Heads mode (the per-head attention products): tile t belongs to head
    // z = t / tiles_per_z, z = b * H + h, and every operand is a 4-D box
    // (k, row, head, sequence) of its tensor map; y of head z starts at
    // b * syb + h * syh with rows ldy apart.  Plain mode: H 1, ldy N.
    int H;
    int tiles_per_z;
    int64_t ldy;
    int64_t syh;
    int64_t syb;
    int causal_tiles;   // tiles whose columns all exceed every row + q_off are not computed
    int causal_k;       // a tile sums only k < (its last row + 1) + q_off
    int q_off;
    int x_head_major;   // 1: x's map orders its dimensions (k, head, row, sequence)
    int w_head_major;
    int w_box_rows;     // w rows per TMA box: the tile's, or fewer when N is narrow
    uint64_t first_wait_ns;   // limit of the MMA thread's first wait (first_wait_limit_ns)
};

struct TileInfo {
    int mb, nb;    // row tile, column tile (within the head)
    int h, b;      // head, sequence (0 in plain mode)
    int kb_end;    // K blocks summed
    bool live;     // false: the tile is skipped by every role
};

// Tile t -> (row tile, column tile): consecutive tiles sweep the column
// tiles of one row tile, so the CTAs in flight share a few rows of x (read
// from HBM once) and the weight matrix, which L2 largely holds.  (Grouping
// 8-32 row tiles per column tile measured no faster on B200: the kernel is
// bound by shared-memory traffic, not by L2 misses.)
template <int BK, bool PAIR, bool HEADS>
__device__ __forceinline__ TileInfo tile_info(int t, const LinearArgs& a)
{
    TileInfo ti;
    int r = t;
    ti.h = ti.b = 0;
    if constexpr (HEADS) {
        const int z = t / a.tiles_per_z;
        r = t - z * a.tiles_per_z;
        ti.b = z / a.H;
        ti.h = z - ti.b * a.H;
    }
    ti.mb = r / a.n_blocks;
    ti.nb = r - ti.mb * a.n_blocks;
    ti.live = true;
    ti.kb_end = a.k_blocks;
    if constexpr (HEADS) {
        // columns (keys) below rows_end are visible to some row of the tile
        const int64_t rows_end = (int64_t)(ti.mb + 1) * LinCfg<BK, PAIR>::tile_rows + a.q_off;
        if (a.causal_tiles && (int64_t)ti.nb * kLinBN >= rows_end) ti.live = false;
        if (a.causal_k && rows_end < a.K) ti.kb_end = (int)((rows_end + BK - 1) / BK);
    }
    return ti;
}

__device__ __forceinline__ float epi_value(float acc, int n, int64_t row, const LinearArgs& a)
{
    float v = acc;
    if (a.bias) v = v + __ldg(a.bias + n);
    if (a.act == GBX_ACT_GELU) v = gelu_tanh(v);
    if (a.resid) v = a.resid[row * a.N + n] + v;
    return v;
}

// 16 accumulator columns of one output row: columns n .. n+15 (n < N).
// yoff: the row's offset in y (row * N in plain mode); the residual is
// always read at row * N + n.
template <bool VEC>
__device__ __forceinline__ void epi_store16(const float (&v)[16], int64_t row, int64_t yoff, int n, const LinearArgs& a)
{
    const int64_t off = row * a.N;
    if (VEC) {
#pragma unroll
        for (int j = 0; j < 16; j += 4) {
            if (n + j >= a.N) break;   // N % 4 == 0: a float4 is all in or all out
            float4 o;
            if (a.bias || a.resid || a.act) {
                float4 b = a.bias ? __ldg(reinterpret_cast<const float4*>(a.bias + n + j)) : make_float4(0.f, 0.f, 0.f, 0.f);
                o = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                if (a.bias) o = add4(o, b);
                if (a.act == GBX_ACT_GELU) o = gelu4(o);
                if (a.resid) o = add4(*reinterpret_cast<const float4*>(a.resid + off + n + j), o);
            } else {
                o = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
            }
            if (a.y_lo) {
                float4 h, l;
                split_value(o.x, h.x, l.x);
                split_value(o.y, h.y, l.y);
                split_value(o.z, h.z, l.z);
                split_value(o.w, h.w, l.w);
                *reinterpret_cast<float4*>(a.y + yoff + n + j) = h;
                *reinterpret_cast<float4*>(a.y_lo + yoff + n + j) = l;
            } else {
                *reinterpret_cast<float4*>(a.y + yoff + n + j) = o;
            }
        }
    } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            if (n + j >= a.N) break;
            const float o = epi_value(v[j], n + j, row, a);
            if (a.y_lo) {
                float h, l;
                split_value(o, h, l);
                a.y[yoff + n + j] = h;
                a.y_lo[yoff + n + j] = l;
            } else {
                a.y[yoff + n + j] = o;
            }
        }
    }
}

// Heads mode, VEC: output columns n .. n+15 of an epilogue warp's 32 rows
// (this lane's row's values v[off .. off+15], off a constant after
// unrolling), written through the warp's
// 32 x 16 staging block `stg`.  Straight from the accumulator's thread-per-row
// layout every warp store would touch 32 rows with 16 bytes each; staged, a
// warp store writes 8 rows x 64 contiguous bytes.  The block is XOR-swizzled
// by 16-byte chunk (chunk ^ ((row >> 1) & 3)), so both the row-wise writes
// and the column-wise reads are free of bank conflicts.  r_rd: the first
// output row this lane writes on the read side (8 rows apart after it),
// out_rd its offset in y plus the lane's 4-column offset.  The heads mode has
// no bias, residual or activation.  All 32 lanes call it.
template <int LEN>
__device__ __forceinline__ void heads_store16(float* stg, int lane, const float (&v)[LEN], int off, int n,
                                              int64_t r_rd, int64_t out_rd, const LinearArgs& a)
{
    float* const wrow = stg + lane * 16;
    const int wsw = (lane >> 1) & 3;
    const int q = lane & 3;
    // the read side's row 8 i + lane / 4 has swizzle (lane >> 3) & 3 for every i
    const float* const rd = stg + (lane >> 2) * 16 + 4 * (q ^ ((lane >> 3) & 3));
    const bool col_ok = n + 4 * q < a.N;
#pragma unroll
    for (int part = 0; part < 2; ++part) {
        if (part == 1 && !a.y_lo) break;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float4 o = make_float4(v[off + 4 * j], v[off + 4 * j + 1], v[off + 4 * j + 2], v[off + 4 * j + 3]);
            if (a.y_lo) {
                float4 h, l;
                split4(o, h, l);
                o = part ? l : h;
            }
            *reinterpret_cast<float4*>(wrow + 4 * (j ^ wsw)) = o;
        }
        __syncwarp();
        float* const dst = (part ? a.y_lo : a.y) + out_rd + n;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float4 o = *reinterpret_cast<const float4*>(rd + 128 * i);
            if (col_ok && r_rd + 8 * i < a.M) *reinterpret_cast<float4*>(dst + 8 * i * a.ldy) = o;
        }
        __syncwarp();
    }
}

template <int BK, bool VEC, bool PAIR, bool HEADS>
__global__ void __launch_bounds__(kLinThreads, 1)
linear_tf32x3_kernel(const __grid_constant__ CUtensorMap map_xh, const __grid_constant__ CUtensorMap map_xl,
                     const __grid_constant__ CUtensorMap map_wh, const __grid_constant__ CUtensorMap map_wl,
                     const LinearArgs a)
{
    using C = LinCfg<BK, PAIR>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::stages * C::stage_bytes);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::nbars);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    // heads mode only (the host adds kLinEpiStageBytes to the launch's shared memory)
    float* const epi_stage = reinterpret_cast<float*>(
        (reinterpret_cast<uintptr_t>(tmem_slot + 2) + 15) & ~uintptr_t(15));
    const uint32_t full0 = tc::smem_u32(bars);                     // full[s]        = full0 + 8 s
    const uint32_t empty0 = full0 + 8 * C::stages;                 // empty[s]
    const uint32_t cfull0 = empty0 + 8 * C::stages;                // chunk_full[b]
    const uint32_t cempty0 = cfull0 + 8 * kLinBuffers;             // chunk_empty[b]
    const uint32_t drain = cempty0 + 8 * kLinBuffers;
    const uint32_t clocal0 = drain + 8;                            // PAIR follower: chunk_empty, local
    const uint32_t smem0 = tc::smem_u32(smem);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // PAIR: the barriers that count both CTAs (full, chunk_empty, drain) live
    // in the leader, rank 0 (chunk_empty counts the leader's epilogue warps
    // and one arrival forwarded for the follower's); empty and chunk_full
    // exist in both (the MMA commit multicasts to the two)
    const uint32_t rank = PAIR ? tc::cluster_rank() : 0;
    const bool leader = rank == 0;
    const int unit = PAIR ? (int)tc::cluster_id_x() : (int)blockIdx.x;        // tile walker
    const int units = PAIR ? (int)tc::cluster_count_x() : (int)gridDim.x;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::stages; ++s) {
            tc::mbar_init(full0 + 8 * s, 1);
            tc::mbar_init(empty0 + 8 * s, 1);
        }
        for (int b = 0; b < kLinBuffers; ++b) {
            tc::mbar_init(cfull0 + 8 * b, 1);
            // one arrival per epilogue warp of this CTA; PAIR: and one
            // forwarded for all of the follower's (see the forwarder below)
            tc::mbar_init(cempty0 + 8 * b, kLinEpiWarps + (PAIR ? 1 : 0));
            tc::mbar_init(clocal0 + 8 * b, kLinEpiWarps);
        }
        tc::mbar_init(drain, 1);
        *abort = 0;
        tc::fence_mbar_init();
        tc::tma_prefetch(&map_xh);
        tc::tma_prefetch(&map_wh);
        if (a.has_xlo) tc::tma_prefetch(&map_xl);
        if (a.has_wlo) tc::tma_prefetch(&map_wl);
    }
    if (warp == 1) {
        if constexpr (PAIR) {
            tc::tmem_alloc_pair(tc::smem_u32(tmem_slot), kLinTmemCols);
            tc::tmem_relinquish_pair();
        } else {
            tc::tmem_alloc(tc::smem_u32(tmem_slot), kLinTmemCols);
            tc::tmem_relinquish();
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if constexpr (PAIR) tc::cluster_sync();   // both CTAs' barriers and TMEM exist before any cross-CTA signal
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------------------------------------------- producer
            const uint32_t cta_bytes =
                (uint32_t)(C::a_bytes * (1 + a.has_xlo) + a.w_box_rows * C::row_bytes * (1 + a.has_wlo));
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued = 0;    // bit s: stage s has had a load issued
            uint32_t lastpar = 0;   // bit s: parity of the phase of its last load
            for (int t = unit; t < a.tiles && !*abort; t += units) {
                const TileInfo ti = tile_info<BK, PAIR, HEADS>(t, a);
                if (!ti.live) continue;
                const int n_left = a.N - ti.nb * kLinBN;
                const int n_mma = n_left >= kLinBN ? kLinBN : (n_left + 15) & ~15;
                const int y_x = ti.mb * C::tile_rows + (int)rank * kLinBM;
                const int y_w = ti.nb * kLinBN + (PAIR ? (int)rank * (n_mma / 2) : 0);
                // 4-D boxes: (k, row, head, sequence), or (k, head, row, sequence)
                const int x1 = a.x_head_major ? ti.h : y_x, x2 = a.x_head_major ? y_x : ti.h;
                const int w1 = a.w_head_major ? ti.h : y_w, w2 = a.w_head_major ? y_w : ti.h;
                for (int kb = 0; kb < ti.kb_end; ++kb) {
                    if (!tc::mbar_wait(empty0 + 8 * stage, phase ^ 1, abort, kLinWaitNs)) break;
                    const uint32_t full = full0 + 8 * stage;
                    const uint32_t base = smem0 + stage * C::stage_bytes;
                    const int x = kb * BK;
                    if constexpr (PAIR && HEADS) {
                        if (leader) tc::mbar_arrive_expect_tx(full, 2 * cta_bytes);
                        const uint32_t fl = tc::mapa(full, 0);
                        tc::tma_load_4d_pair(base, &map_xh, fl, x, x1, x2, ti.b);
                        if (a.has_xlo) tc::tma_load_4d_pair(base + C::a_bytes, &map_xl, fl, x, x1, x2, ti.b);
                        tc::tma_load_4d_pair(base + 2 * C::a_bytes, &map_wh, fl, x, w1, w2, ti.b);
                        if (a.has_wlo)
                            tc::tma_load_4d_pair(base + 2 * C::a_bytes + C::b_bytes, &map_wl, fl, x, w1, w2, ti.b);
                    } else if constexpr (HEADS) {
                        tc::mbar_arrive_expect_tx(full, cta_bytes);
                        tc::tma_load_4d(base, &map_xh, full, x, x1, x2, ti.b);
                        if (a.has_xlo) tc::tma_load_4d(base + C::a_bytes, &map_xl, full, x, x1, x2, ti.b);
                        tc::tma_load_4d(base + 2 * C::a_bytes, &map_wh, full, x, w1, w2, ti.b);
                        if (a.has_wlo) tc::tma_load_4d(base + 2 * C::a_bytes + C::b_bytes, &map_wl, full, x, w1, w2, ti.b);
                    } else if constexpr (PAIR) {
                        if (leader) tc::mbar_arrive_expect_tx(full, 2 * cta_bytes);   // both CTAs' tiles
                        const uint32_t fl = tc::mapa(full, 0);
                        tc::tma_load_2d_pair(base, &map_xh, fl, x, y_x);
                        if (a.has_xlo) tc::tma_load_2d_pair(base + C::a_bytes, &map_xl, fl, x, y_x);
                        tc::tma_load_2d_pair(base + 2 * C::a_bytes, &map_wh, fl, x, y_w);
                        if (a.has_wlo) tc::tma_load_2d_pair(base + 2 * C::a_bytes + C::b_bytes, &map_wl, fl, x, y_w);
                    } else {
                        tc::mbar_arrive_expect_tx(full, cta_bytes);
                        tc::tma_load_2d(base, &map_xh, full, x, y_x);
                        if (a.has_xlo) tc::tma_load_2d(base + C::a_bytes, &map_xl, full, x, y_x);
                        tc::tma_load_2d(base + 2 * C::a_bytes, &map_wh, full, x, y_w);
                        if (a.has_wlo) tc::tma_load_2d(base + 2 * C::a_bytes + C::b_bytes, &map_wl, full, x, y_w);
                    }
                    issued |= 1u << stage;
                    lastpar = (lastpar & ~(1u << stage)) | (phase << stage);
                    if (++stage == C::stages) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            // Every load issued has landed before the CTA may exit.  PAIR: the
            // leader's full barriers count both CTAs' loads; the follower's
            // last loads are consumed by the leader's MMAs before the final
            // cluster barrier (or, after an abort, had a wait limit's time to land).
            if (leader)
                for (int s = 0; s < C::stages; ++s)
                    if (issued & (1u << s)) tc::mbar_wait(full0 + 8 * s, (lastpar >> s) & 1, nullptr, kLinWaitNs);
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            // ---------------------------------------------------- MMA issuer
            int stage = 0;
            uint32_t phase = 0;
            int buf = 0;
            uint32_t buf_phase = 0;
            bool ok = true;
            bool first = true;   // the first wait on a load takes a.first_wait_ns (0: give up at once)
            for (int t = unit; t < a.tiles && ok; t += units) {
                // the last column tile runs only as wide as N needs (a multiple of 16)
                const TileInfo ti = tile_info<BK, PAIR, HEADS>(t, a);
                if (!ti.live) continue;
                const int n_left = a.N - ti.nb * kLinBN;
                const int n_mma = n_left >= kLinBN ? kLinBN : (n_left + 15) & ~15;
                const uint32_t idesc = tc::idesc_tf32(C::tile_rows, n_mma);
                const int chunks = (ti.kb_end + C::chunk_blocks - 1) / C::chunk_blocks;
                for (int c = 0; c < chunks && ok; ++c) {
                    if (!tc::mbar_wait(cempty0 + 8 * buf, buf_phase ^ 1, abort, kLinWaitNs)) {
                        ok = false;
                        break;
                    }
                    tc::fence_after_sync();
                    const uint32_t d = tmem + buf * kLinBN;
                    const int kb0 = c * C::chunk_blocks;
                    const int kb1 = kb0 + C::chunk_blocks < ti.kb_end ? kb0 + C::chunk_blocks : ti.kb_end;
                    for (int kb = kb0; kb < kb1; ++kb) {
                        const uint64_t limit = first ? a.first_wait_ns : kLinWaitNs;
                        first = false;
                        if (limit == 0) *abort = 1;
                        if (limit == 0 || !tc::mbar_wait(full0 + 8 * stage, phase, abort, limit)) {
                            ok = false;
                            break;
                        }
                        tc::fence_after_sync();
                        const uint32_t base = smem0 + stage * C::stage_bytes;
#pragma unroll
                        for (int ks = 0; ks < C::ksteps; ++ks) {
                            const uint32_t off = ks * 32;
                            const uint64_t xh = tc::smem_desc(base + off, C::row_bytes);
                            const uint64_t wh = tc::smem_desc(base + 2 * C::a_bytes + off, C::row_bytes);
                            const uint32_t acc0 = (kb != kb0) | (ks != 0);
                            if constexpr (PAIR) {
                                tc::mma_tf32_pair(d, xh, wh, idesc, acc0);
                                if (a.has_wlo)
                                    tc::mma_tf32_pair(
                                        d, xh, tc::smem_desc(base + 2 * C::a_bytes + C::b_bytes + off, C::row_bytes),
                                        idesc, 1);
                                if (a.has_xlo)
                                    tc::mma_tf32_pair(d, tc::smem_desc(base + C::a_bytes + off, C::row_bytes), wh,
                                                      idesc, 1);
                            } else {
                                tc::mma_tf32(d, xh, wh, idesc, acc0);
                                if (a.has_wlo)
                                    tc::mma_tf32(d, xh,
                                                 tc::smem_desc(base + 2 * C::a_bytes + C::b_bytes + off, C::row_bytes),
                                                 idesc, 1);
                                if (a.has_xlo)
                                    tc::mma_tf32(d, tc::smem_desc(base + C::a_bytes + off, C::row_bytes), wh, idesc,
                                                 1);
                            }
                        }
                        // the stage is free (in both CTAs) once these MMAs are done
                        if constexpr (PAIR)
                            tc::mma_commit_pair_multicast(empty0 + 8 * stage, 3);
                        else
                            tc::mma_commit(empty0 + 8 * stage);
                        if (++stage == C::stages) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                    if (!ok) break;
                    // chunk complete (in both CTAs' TMEM)
                    if constexpr (PAIR)
                        tc::mma_commit_pair_multicast(cfull0 + 8 * buf, 3);
                    else
                        tc::mma_commit(cfull0 + 8 * buf);
                    if (++buf == kLinBuffers) {
                        buf = 0;
                        buf_phase ^= 1;
                    }
                }
            }
            // every MMA issued has completed before TMEM is freed
            if constexpr (PAIR)
                tc::mma_commit_pair(drain);
            else
                tc::mma_commit(drain);
            tc::mbar_wait(drain, 0, nullptr, kLinWaitNs);
        } else if (PAIR && lane == 0) {
            // ---------------------------------------------------- forwarder
            // The follower's epilogue warps release each chunk buffer on
            // their own CTA's barrier; this thread, which has no global
            // stores in flight, passes one cluster-scope arrival on to the
            // leader's chunk_empty.  (A cluster-scope release from an
            // epilogue warp would first wait for that warp's output stores
            // to drain.)
            int buf = 0;
            uint32_t buf_phase = 0;
            bool ok = true;
            for (int t = unit; t < a.tiles && ok; t += units) {
                const TileInfo ti = tile_info<BK, PAIR, HEADS>(t, a);
                if (!ti.live) continue;
                const int chunks = (ti.kb_end + C::chunk_blocks - 1) / C::chunk_blocks;
                for (int c = 0; c < chunks; ++c) {
                    if (!tc::mbar_wait(clocal0 + 8 * buf, buf_phase, abort, kLinWaitNs)) {
                        ok = false;
                        break;
                    }
                    tc::mbar_arrive_cluster(tc::mapa(cempty0 + 8 * buf, 0));
                    if (++buf == kLinBuffers) {
                        buf = 0;
                        buf_phase ^= 1;
                    }
                }
            }
        }
    } else {
        // -------------------------------------------------------- epilogue
        const int quarter = warp & 3;   // the TMEM lanes this warp may read
        const int col0 = ((warp - 2) >> 2) * kLinEpiCols;
        const int row_in_tile = (int)rank * kLinBM + 32 * quarter + lane;
        int buf = 0;
        uint32_t buf_phase = 0;
        bool ok = true;
        for (int t = unit; t < a.tiles && ok; t += units) {
            const TileInfo ti = tile_info<BK, PAIR, HEADS>(t, a);
            if (!ti.live) continue;
            const int mb = ti.mb, nb = ti.nb;
            const int chunks = (ti.kb_end + C::chunk_blocks - 1) / C::chunk_blocks;
            // heads mode: per-warp output geometry of the staged stores
            float* const stg = epi_stage + (warp - 2) * kLinStageFloats;
            const int64_t r_rd = (int64_t)mb * C::tile_rows + (int)rank * kLinBM + 32 * quarter + (lane >> 2);
            const int64_t out_rd = (int64_t)ti.b * a.syb + (int64_t)ti.h * a.syh + r_rd * a.ldy + 4 * (lane & 3);
            const int n0 = nb * kLinBN + col0;
            if (HEADS && VEC && chunks == 1) {
                // one K chunk (a head-wide K): stream TMEM to the output 32
                // columns at a time instead of holding the row in registers
                const bool ready = tc::mbar_wait(cfull0 + 8 * buf, buf_phase, abort, kLinWaitNs);
                if (!__all_sync(0xffffffffu, ready)) {
                    ok = false;
                    break;
                }
                tc::fence_after_sync();
                const uint32_t tbase = tmem + ((uint32_t)(32 * quarter) << 16) + buf * kLinBN + col0;
#pragma unroll 1
                for (int g = 0; g < kLinEpiCols / 32; ++g) {
                    if (n0 + 32 * g >= a.N) break;   // uniform over the warp
                    float v[32];
                    tc::tmem_ld32(tbase + 32 * g, v);
                    tc::tmem_ld_wait();
                    heads_store16(stg, lane, v, 0, n0 + 32 * g, r_rd, out_rd, a);
                    if (n0 + 32 * g + 16 < a.N) heads_store16(stg, lane, v, 16, n0 + 32 * g + 16, r_rd, out_rd, a);
                }
                tc::fence_before_sync();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive((PAIR && !leader ? clocal0 : cempty0) + 8 * buf);
                if (++buf == kLinBuffers) {
                    buf = 0;
                    buf_phase ^= 1;
                }
                continue;
            }
            float acc[kLinEpiCols];
#pragma unroll
            for (int j = 0; j < kLinEpiCols; ++j) acc[j] = 0.0f;
            for (int c = 0; c < chunks; ++c) {
                // warp-uniform outcome: tcgen05.ld below needs the whole warp
                const bool ready = tc::mbar_wait(cfull0 + 8 * buf, buf_phase, abort, kLinWaitNs);
                if (!__all_sync(0xffffffffu, ready)) {
                    ok = false;
                    break;
                }
                tc::fence_after_sync();
                const uint32_t tbase = tmem + ((uint32_t)(32 * quarter) << 16) + buf * kLinBN + col0;
                const int n_left = a.N - nb * kLinBN - col0;   // columns of this warp below N
#pragma unroll
                for (int g = 0; g < kLinEpiCols / 32; ++g) {
                    if (32 * g < n_left) {   // uniform over the warp
                        float v[32];
                        tc::tmem_ld32(tbase + 32 * g, v);
                        tc::tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 32; ++i) acc[32 * g + i] += v[i];
                    }
                }
                tc::fence_before_sync();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive((PAIR && !leader ? clocal0 : cempty0) + 8 * buf);
                if (++buf == kLinBuffers) {
                    buf = 0;
                    buf_phase ^= 1;
                }
            }
            if (!ok) break;
            const int64_t row = (int64_t)mb * C::tile_rows + row_in_tile;
            int64_t yoff = row * a.ldy;
            if constexpr (HEADS) yoff += ti.b * a.syb + ti.h * a.syh;
            if constexpr (HEADS && VEC) {
#pragma unroll
                for (int g = 0; g < kLinEpiCols / 16; ++g) {
                    if (n0 + 16 * g >= a.N) break;   // uniform over the warp
                    heads_store16(stg, lane, acc, 16 * g, n0 + 16 * g, r_rd, out_rd, a);
                }
            } else if (row < a.M) {
#pragma unroll
                for (int g = 0; g < kLinEpiCols / 16; ++g) {
                    if (n0 + 16 * g < a.N) {
                        float v[16];
#pragma unroll
                        for (int i = 0; i < 16; ++i) v[i] = acc[16 * g + i];
                        epi_store16<VEC>(v, row, yoff, n0 + 16 * g, a);
                    }
                }
            }
        }
    }

    __syncthreads();   // every role has left its loop (all waits are bounded)
    if constexpr (PAIR) tc::cluster_sync();   // the leader's MMAs, which read both CTAs, are drained
    if (warp == 1) {
        __syncwarp();
        tc::fence_after_sync();
        if constexpr (PAIR)
            tc::tmem_dealloc_pair(tmem, kLinTmemCols);
        else
            tc::tmem_dealloc(tmem, kLinTmemCols);
    }
    if (threadIdx.x == 0 && *abort && a.err) atomicOr(a.err, GBX_LINEAR_TIMEOUT);
}

// General path (K not a multiple of 4, or operands off 16-byte alignment):
// one thread per output on the CUDA cores, the same three product terms
// with fp32 FMAs, the same epilogue.
__global__ void __launch_bounds__(256)
linear_general_kernel(const float* __restrict__ xh, const float* __restrict__ xl, const float* __restrict__ wh,
                      const float* __restrict__ wl, const LinearArgs a)
{
    const int64_t total = a.M * a.N;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t m = i / a.N;
        const int n = (int)(i - m * a.N);
        const float* xr = xh + m * a.K;
        const float* wr = wh + (int64_t)n * a.K;
        float acc = 0.0f;
        for (int k = 0; k < a.K; ++k) {
            acc = fmaf(xr[k], wr[k], acc);
            if (wl) acc = fmaf(xr[k], wl[(int64_t)n * a.K + k], acc);
            if (xl) acc = fmaf(xl[m * a.K + k], wr[k], acc);
        }
        const float o = epi_value(acc, n, m, a);
        if (a.y_lo) {
            float h, l;
            split_value(o, h, l);
            a.y[i] = h;
            a.y_lo[i] = l;
        } else {
            a.y[i] = o;
        }
    }
}

// An operand of the heads mode: element (sequence b, head h, row r, k) at
// base[b * sb + h * sh + r * ld + k], in elements.  head_major orders the
// tensor map's dimensions (k, head, row, sequence) instead of (k, row, head,
// sequence), so that the strides increase with the dimension (the Q and K
// column blocks of a [tokens, 3d] QKV buffer: sh = hd < ld).
struct HeadsOperand {
    const float* hi;
    const float* lo;
    int64_t ld, sh, sb;
    int rows;
    bool head_major;
};

// General path of the heads mode (operands the tensor maps cannot describe):
// one thread per output, the same three product terms, the same causal
// limits at element granularity (outputs past the diagonal are not written).
__global__ void __launch_bounds__(256)
linear_heads_general_kernel(const HeadsOperand x, const HeadsOperand w, const LinearArgs a, int B)
{
    const int64_t per_z = a.M * (int64_t)a.N;
    const int64_t total = per_z * a.H * B;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t z = i / per_z;
        const int64_t r = i - z * per_z;
        const int64_t m = r / a.N;
        const int n = (int)(r - m * a.N);
        const int64_t b = z / a.H, h = z - b * a.H;
        if (a.causal_tiles && n > m + a.q_off) continue;
        const int64_t kend = a.causal_k ? (m + a.q_off + 1 < a.K ? m + a.q_off + 1 : a.K) : a.K;
        const int64_t xo = b * x.sb + h * x.sh + m * x.ld, wo = b * w.sb + h * w.sh + (int64_t)n * w.ld;
        float acc = 0.0f;
        for (int64_t k = 0; k < kend; ++k) {
            acc = fmaf(x.hi[xo + k], w.hi[wo + k], acc);
            if (w.lo) acc = fmaf(x.hi[xo + k], w.lo[wo + k], acc);
            if (x.lo) acc = fmaf(x.lo[xo + k], w.hi[wo + k], acc);
        }
        const int64_t yo = b * a.syb + h * a.syh + m * a.ldy + n;
        if (a.y_lo) {
            float hv, lv;
            split_value(acc, hv, lv);
            a.y[yo] = hv;
            a.y_lo[yo] = lv;
        } else {
            a.y[yo] = acc;
        }
    }
}

// vt[((b * H + h) * hd + i) * S + s] = v[(b * S + s) * ld + h * hd + i]:
// the V block of each head transposed so that the attention output's
// contraction index (the key position) is contiguous, as the tensor maps
// read it.  32 x 32 tiles through shared memory; coalesced on both sides.
__global__ void __launch_bounds__(256)
transpose_heads_kernel(const float* __restrict__ v, int64_t ld, float* __restrict__ vt, int S, int H, int hd)
{
    __shared__ float tile[32][33];
    const int z = blockIdx.z;
    const int b = z / H, h = z - b * H;
    const int s0 = blockIdx.x * 32, i0 = blockIdx.y * 32;
    const float* src = v + (int64_t)b * S * ld + (int64_t)h * hd;
    for (int r = threadIdx.y; r < 32; r += 8) {
        const int sp = s0 + r, i = i0 + threadIdx.x;
        if (sp < S && i < hd) tile[r][threadIdx.x] = src[(int64_t)sp * ld + i];
    }
    __syncthreads();
    float* dst = vt + (int64_t)z * hd * S;
    for (int r = threadIdx.y; r < 32; r += 8) {
        const int i = i0 + r, sp = s0 + threadIdx.x;
        if (i < hd && sp < S) dst[(int64_t)i * S + sp] = tile[threadIdx.x][r];
    }
}

// ------------------------------------------------------------------ split
__global__ void __launch_bounds__(256) split_tf32_vec_kernel(const float4* x, float4* hi, float4* lo, int64_t n4)
{
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
        const float4 v = x[i];
        float4 h, l;
        split_value(v.x, h.x, l.x);
        split_value(v.y, h.y, l.y);
        split_value(v.z, h.z, l.z);
        split_value(v.w, h.w, l.w);
        hi[i] = h;
        lo[i] = l;
    }
}

__global__ void __launch_bounds__(256) split_tf32_scalar_kernel(const float* x, float* hi, float* lo, int64_t n)
{
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        float h, l;
        split_value(x[i], h, l);
        hi[i] = h;
        lo[i] = l;
    }
}

// ------------------------------------------------------------------ host
// Row-major [rows, K] fp32, boxes of box_rows x BK with the BK-wide swizzle.
static int make_map(CUtensorMap* m, const float* base, int64_t rows, int K, int box_rows, int BK)
{
    EncodeTiledFn fn = encode_tiled();
    if (!fn) return set_error(GBX_ECUDA, "gbx_linear: cuTensorMapEncodeTiled unavailable from the driver");
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)K * sizeof(float)};
    const cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE,
                          BK == 32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(GBX_EINVAL, "gbx_linear: tensor map rejected (CUresult %d)", (int)r);
    return GBX_OK;
}

// One plane (hi or lo) of a heads-mode operand as a 4-D map, boxes of
// BK x box_rows (one head, one sequence) with the BK-wide swizzle.
static int make_map4(CUtensorMap* m, const float* base, const HeadsOperand& op, int K, int H, int B, int box_rows,
                     int BK)
{
    EncodeTiledFn fn = encode_tiled();
    if (!fn) return set_error(GBX_ECUDA, "gbx_attn: cuTensorMapEncodeTiled unavailable from the driver");
    const cuuint64_t e = sizeof(float);
    cuuint64_t dims[4], strides[3];
    cuuint32_t box[4];
    dims[0] = (cuuint64_t)K;
    dims[3] = (cuuint64_t)B;
    strides[2] = (cuuint64_t)op.sb * e;
    box[0] = (cuuint32_t)BK;
    box[3] = 1;
    if (op.head_major) {
        dims[1] = (cuuint64_t)H;
        dims[2] = (cuuint64_t)op.rows;
        strides[0] = (cuuint64_t)op.sh * e;
        strides[1] = (cuuint64_t)op.ld * e;
        box[1] = 1;
        box[2] = (cuuint32_t)box_rows;
    } else {
        dims[1] = (cuuint64_t)op.rows;
        dims[2] = (cuuint64_t)H;
        strides[0] = (cuuint64_t)op.ld * e;
        strides[1] = (cuuint64_t)op.sh * e;
        box[1] = (cuuint32_t)box_rows;
        box[2] = 1;
    }
    if (B == 1) strides[2] = strides[1] * dims[2];   // unused; any valid stride
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE,
                          BK == 32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(GBX_EINVAL, "gbx_attn: tensor map rejected (CUresult %d)", (int)r);
    return GBX_OK;
}

// hx / hw: the heads-mode operands (HEADS only; B sequences of a.H heads).
template <int BK, bool VEC, bool PAIR, bool HEADS>
static int launch_linear(const float* x_hi, const float* x_lo, const float* w_hi, const float* w_lo, LinearArgs a,
                         cudaStream_t s, const HeadsOperand* hx = nullptr, const HeadsOperand* hw = nullptr, int B = 1)
{
    using C = LinCfg<BK, PAIR>;
    const size_t smem = C::smem + (HEADS ? kLinEpiStageBytes : 0);
    DeviceInfo di;
    if (device_info(&di) != GBX_OK) return GBX_ECUDA;
    if ((size_t)di.max_smem_optin < smem)
        return set_error(GBX_ERANGE, "gbx_linear: needs %zu bytes of shared memory per CTA", smem);
    const int64_t m_blocks = (a.M + C::tile_rows - 1) / C::tile_rows;
    const int64_t zs = HEADS ? (int64_t)a.H * B : 1;
    if (m_blocks * a.n_blocks * zs > 0x7fffffffLL) return set_error(GBX_ERANGE, "gbx_linear: too many tiles");
    a.m_blocks = (int)m_blocks;
    a.tiles_per_z = (int)(m_blocks * a.n_blocks);
    a.tiles = (int)(m_blocks * a.n_blocks * zs);
    a.k_blocks = (a.K + BK - 1) / BK;
    a.w_box_rows = C::b_rows;
    a.first_wait_ns = first_wait_limit_ns();
    if (HEADS && a.n_blocks == 1) {   // a narrow N (a head's width): load only the rows the MMA reads
        const int n16 = (a.N + 15) & ~15;
        const int rows = PAIR ? n16 / 2 : n16;
        if (rows < a.w_box_rows) a.w_box_rows = rows;
    }
    CUtensorMap mxh, mxl, mwh, mwl;
    int rc;
    if constexpr (HEADS) {
        if ((rc = make_map4(&mxh, hx->hi, *hx, a.K, a.H, B, C::a_rows, BK)) != GBX_OK) return rc;
        if ((rc = make_map4(&mwh, hw->hi, *hw, a.K, a.H, B, a.w_box_rows, BK)) != GBX_OK) return rc;
        mxl = mxh;
        mwl = mwh;
        if (a.has_xlo && (rc = make_map4(&mxl, hx->lo, *hx, a.K, a.H, B, C::a_rows, BK)) != GBX_OK) return rc;
        if (a.has_wlo && (rc = make_map4(&mwl, hw->lo, *hw, a.K, a.H, B, a.w_box_rows, BK)) != GBX_OK) return rc;
    } else {
        if ((rc = make_map(&mxh, x_hi, a.M, a.K, C::a_rows, BK)) != GBX_OK) return rc;
        if ((rc = make_map(&mwh, w_hi, a.N, a.K, C::b_rows, BK)) != GBX_OK) return rc;
        if (a.has_xlo) {
            if ((rc = make_map(&mxl, x_lo, a.M, a.K, C::a_rows, BK)) != GBX_OK) return rc;
        } else {
            mxl = mxh;   // never loaded
        }
        if (a.has_wlo) {
            if ((rc = make_map(&mwl, w_lo, a.N, a.K, C::b_rows, BK)) != GBX_OK) return rc;
        } else {
            mwl = mwh;
        }
    }
    auto k = linear_tf32x3_kernel<BK, VEC, PAIR, HEADS>;
    // per device, so set on every call (a host-side attribute write)
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return set_error(GBX_ECUDA, "gbx_linear: shared-memory attribute refused");
    if constexpr (!PAIR) {
        const int grid = a.tiles < di.sm_count ? a.tiles : di.sm_count;
        k<<<grid, kLinThreads, smem, s>>>(mxh, mxl, mwh, mwl, a);
        return check_launch("gbx_linear");
    } else {
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.blockDim = dim3(kLinThreads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = s;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        cfg.gridDim = dim3(2 * (unsigned)(di.sm_count / 2));
        int clusters = 0;
        if (cudaOccupancyMaxActiveClusters(&clusters, k, &cfg) != cudaSuccess || clusters < 1)
            return set_error(GBX_ECUDA, "gbx_linear: no resident CTA pair fits");
        if (clusters > a.tiles) clusters = a.tiles;
        cfg.gridDim = dim3(2 * (unsigned)clusters);
        if (cudaLaunchKernelEx(&cfg, k, mxh, mxl, mwh, mwl, a) != cudaSuccess)
            return set_error(GBX_ECUDA, "gbx_linear: cluster launch failed: %s", cudaGetErrorString(cudaGetLastError()));
        return check_launch("gbx_linear");
    }
}

}  // namespace gbx

using namespace gbx;

extern "C" int gbx_split_tf32(const float* x, float* hi, float* lo, int64_t n, gbx_stream_t stream)
{
    if (n < 0) return set_error(GBX_EINVAL, "gbx_split_tf32: n=%lld", (long long)n);
    if (n == 0) return GBX_OK;
    if (!x || !hi || !lo) return set_error(GBX_EINVAL, "gbx_split_tf32: null pointer");
    if (lo == x || lo == hi) return set_error(GBX_EINVAL, "gbx_split_tf32: lo must not alias x or hi");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (n % 4 == 0 && aligned16(x) && aligned16(hi) && aligned16(lo)) {
        const int grid = persistent_grid(split_tf32_vec_kernel, 256, 0, (n / 4 + 255) / 256, 8);
        if (grid < 1) return GBX_ECUDA;
        split_tf32_vec_kernel<<<grid, 256, 0, s>>>(reinterpret_cast<const float4*>(x), reinterpret_cast<float4*>(hi),
                                                   reinterpret_cast<float4*>(lo), n / 4);
    } else {
        const int grid = persistent_grid(split_tf32_scalar_kernel, 256, 0, (n + 255) / 256, 8);
        if (grid < 1) return GBX_ECUDA;
        split_tf32_scalar_kernel<<<grid, 256, 0, s>>>(x, hi, lo, n);
    }
    return check_launch("gbx_split_tf32");
}

// Tile K width: 16 (64-byte rows, 4 pipeline stages; 6 in CTA pairs) unless
// gbx_linear_set_tiles selects 32 (128-byte rows).  CTA pairs (M 256 tiles
// over two SMs) for M >= kLinPairMinRows unless gbx_linear_set_tiles turns
// them off (0) or on for every shape (1).  Process-wide, read at each launch.
constexpr int64_t kLinPairMinRows = 1024;
constexpr int kLinMaxSplit = 16;   // K slices of gbx_linear_splitk

static std::atomic<int> g_lin_bk{16};
static std::atomic<int> g_lin_pair{-1};   // -1 auto, 0 never, 1 always

static int linear_bk() { return g_lin_bk.load(std::memory_order_relaxed); }
static int linear_pair_mode() { return g_lin_pair.load(std::memory_order_relaxed); }

extern "C" int gbx_linear_set_tiles(int k_block, int pair_mode, int* prev_k_block, int* prev_pair_mode)
{
    if (k_block != 16 && k_block != 32) return set_error(GBX_EINVAL, "gbx_linear_set_tiles: k_block=%d", k_block);
    if (pair_mode < -1 || pair_mode > 1)
        return set_error(GBX_EINVAL, "gbx_linear_set_tiles: pair_mode=%d", pair_mode);
    const int pk = g_lin_bk.exchange(k_block), pp = g_lin_pair.exchange(pair_mode);
    if (prev_k_block) *prev_k_block = pk;
    if (prev_pair_mode) *prev_pair_mode = pp;
    return GBX_OK;
}

extern "C" int gbx_linear(const float* x_hi, const float* x_lo, const float* w_hi, const float* w_lo,
                          const float* bias, const float* resid, float* y, float* y_lo, int64_t M, int N, int K,
                          int act, int* err_flag, gbx_stream_t stream)
{
    if (M < 0 || N <= 0 || K <= 0)
        return set_error(GBX_EINVAL, "gbx_linear: M=%lld N=%d K=%d", (long long)M, N, K);
    if (M == 0) return GBX_OK;
    if (!x_hi || !w_hi || !y) return set_error(GBX_EINVAL, "gbx_linear: null pointer");
    if (act != GBX_ACT_NONE && act != GBX_ACT_GELU) return set_error(GBX_EINVAL, "gbx_linear: act=%d", act);
    if (y_lo == y || (const float*)y == x_hi || (const float*)y == w_hi || (x_lo && (const float*)y == x_lo) ||
        (w_lo && (const float*)y == w_lo))
        return set_error(GBX_EINVAL, "gbx_linear: y aliases an operand");
    if (M > 0x7fffffffLL) return set_error(GBX_ERANGE, "gbx_linear: M=%lld", (long long)M);
    const int64_t n_blocks = ((int64_t)N + kLinBN - 1) / kLinBN;

    LinearArgs a;
    a.bias = bias;
    a.resid = resid;
    a.y = y;
    a.y_lo = y_lo;
    a.err = err_flag;
    a.M = M;
    a.N = N;
    a.K = K;
    a.n_blocks = (int)n_blocks;
    a.act = act;
    a.has_xlo = x_lo != nullptr;
    a.has_wlo = w_lo != nullptr;
    a.H = 1;
    a.ldy = N;
    a.syh = a.syb = 0;
    a.causal_tiles = a.causal_k = a.q_off = 0;
    a.x_head_major = a.w_head_major = 0;
    const bool vec = N % 4 == 0 && aligned16(y) && (!y_lo || aligned16(y_lo)) && (!resid || aligned16(resid)) &&
                     (!bias || aligned16(bias));
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const bool tma_ok = K % 4 == 0 && aligned16(x_hi) && aligned16(w_hi) && (!x_lo || aligned16(x_lo)) &&
                        (!w_lo || aligned16(w_lo));
    if (!tma_ok) {
        a.m_blocks = a.tiles = a.k_blocks = a.tiles_per_z = a.w_box_rows = 0;   // unused by the general kernel
        const int grid = persistent_grid(linear_general_kernel, 256, 0, (M * N + 255) / 256, 8);
        if (grid < 1) return GBX_ECUDA;
        linear_general_kernel<<<grid, 256, 0, s>>>(x_hi, x_lo, w_hi, w_lo, a);
        return check_launch("gbx_linear");
    }
    const int pm = linear_pair_mode();
    const bool pair = pm == 1 || (pm != 0 && M >= kLinPairMinRows);
#define GBX_LIN(BKV, VECV, PAIRV) launch_linear<BKV, VECV, PAIRV, false>(x_hi, x_lo, w_hi, w_lo, a, s)
    if (linear_bk() == 32) {
        if (pair) return vec ? GBX_LIN(32, true, true) : GBX_LIN(32, false, true);
        return vec ? GBX_LIN(32, true, false) : GBX_LIN(32, false, false);
    }
    if (pair) return vec ? GBX_LIN(16, true, true) : GBX_LIN(16, false, true);
    return vec ? GBX_LIN(16, true, false) : GBX_LIN(16, false, false);
#undef GBX_LIN
}

// ------------------------------------------------------------------ attention
// y[z] = x[z] . w[z]^T for every head z = b * H + h of B sequences, on the
// heads mode of the tensor-core kernel (or its general path).
// bk: the K block, 16 (64-byte swizzled rows) or 32 (128-byte rows; P.V
// measured 6% faster with it on B200, its P rows being a long K stream)
static int heads_gemm(const char* what, const HeadsOperand& x, const HeadsOperand& w, float* y, float* y_lo,
                      int64_t ldy, int64_t syh, int64_t syb, int B, int H, int M, int N, int K, int causal_tiles,
                      int causal_k, int* err_flag, cudaStream_t s, int bk = 16)
{
    LinearArgs a;
    a.bias = nullptr;
    a.resid = nullptr;
    a.y = y;
    a.y_lo = y_lo;
    a.err = err_flag;
    a.M = M;
    a.N = N;
    a.K = K;
    a.n_blocks = (N + kLinBN - 1) / kLinBN;
    a.act = GBX_ACT_NONE;
    a.has_xlo = x.lo != nullptr;
    a.has_wlo = w.lo != nullptr;
    a.H = H;
    a.ldy = ldy;
    a.syh = syh;
    a.syb = syb;
    a.causal_tiles = causal_tiles;
    a.causal_k = causal_k;
    a.q_off = 0;
    a.x_head_major = x.head_major;
    a.w_head_major = w.head_major;
    auto al16 = [](const void* p) { return p == nullptr || aligned16(p); };
    auto st4 = [](const HeadsOperand& o) { return o.ld % 4 == 0 && o.sh % 4 == 0 && o.sb % 4 == 0; };
    const bool tma_ok = K % 4 == 0 && st4(x) && st4(w) && al16(x.hi) && al16(x.lo) && al16(w.hi) && al16(w.lo);
    const bool vec = N % 4 == 0 && ldy % 4 == 0 && syh % 4 == 0 && syb % 4 == 0 && al16(y) && al16(y_lo);
    if (!tma_ok) {
        a.m_blocks = a.tiles = a.k_blocks = a.tiles_per_z = a.w_box_rows = 0;
        const int64_t total = (int64_t)B * H * M * N;
        const int grid = persistent_grid(linear_heads_general_kernel, 256, 0, (total + 255) / 256, 8);
        if (grid < 1) return GBX_ECUDA;
        linear_heads_general_kernel<<<grid, 256, 0, s>>>(x, w, a, B);
        return check_launch(what);
    }
    const int pm = linear_pair_mode();
    const bool pair = pm == 1 || (pm != 0 && M >= kLinPairMinRows);
#define GBX_HEADS(BKV, VECV, PAIRV) launch_linear<BKV, VECV, PAIRV, true>(x.hi, x.lo, w.hi, w.lo, a, s, &x, &w, B)
    if (bk == 32) {
        if (pair) return vec ? GBX_HEADS(32, true, true) : GBX_HEADS(32, false, true);
        return vec ? GBX_HEADS(32, true, false) : GBX_HEADS(32, false, false);
    }
    if (pair) return vec ? GBX_HEADS(16, true, true) : GBX_HEADS(16, false, true);
    return vec ? GBX_HEADS(16, true, false) : GBX_HEADS(16, false, false);
#undef GBX_HEADS
}

static int heads_dims(const char* what, int B, int S, int H, int hd)
{
    if (B <= 0 || S <= 0 || H <= 0 || hd <= 0) return set_error(GBX_EINVAL, "%s: B=%d S=%d H=%d hd=%d", what, B, S, H, hd);
    if ((int64_t)B * H * S * S > ((int64_t)1 << 40) || (int64_t)B * H > 65535)
        return set_error(GBX_ERANGE, "%s: B=%d H=%d S=%d too large", what, B, H, S);
    return GBX_OK;
}

extern "C" int gbx_attn_scores(const float* q_hi, const float* q_lo, const float* k_hi, const float* k_lo, int64_t ld,
                               float* dots, int B, int S, int H, int hd, int causal, int* err_flag,
                               gbx_stream_t stream)
{
    if (int rc = heads_dims("gbx_attn_scores", B, S, H, hd)) return rc;
    if (ld < (int64_t)H * hd) return set_error(GBX_EINVAL, "gbx_attn_scores: ld=%lld < H*hd", (long long)ld);
    if (!q_hi || !k_hi || !dots) return set_error(GBX_EINVAL, "gbx_attn_scores: null pointer");
    if ((const float*)dots == q_hi || (const float*)dots == k_hi || (q_lo && (const float*)dots == q_lo) ||
        (k_lo && (const float*)dots == k_lo))
        return set_error(GBX_EINVAL, "gbx_attn_scores: dots aliases an operand");
    const HeadsOperand x{q_hi, q_lo, ld, hd, (int64_t)S * ld, S, true};
    const HeadsOperand w{k_hi, k_lo, ld, hd, (int64_t)S * ld, S, true};
    return heads_gemm("gbx_attn_scores", x, w, dots, nullptr, S, (int64_t)S * S, (int64_t)H * S * S, B, H, S, S, hd,
                      causal ? 1 : 0, 0, err_flag, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int gbx_attn_values(const float* p_hi, const float* p_lo, const float* vt_hi, const float* vt_lo,
                               float* out, float* out_lo, int64_t ld_out, int B, int S, int H, int hd, int causal,
                               int* err_flag, gbx_stream_t stream)
{
    if (int rc = heads_dims("gbx_attn_values", B, S, H, hd)) return rc;
    if (ld_out < (int64_t)H * hd) return set_error(GBX_EINVAL, "gbx_attn_values: ld_out=%lld < H*hd", (long long)ld_out);
    if (!p_hi || !vt_hi || !out) return set_error(GBX_EINVAL, "gbx_attn_values: null pointer");
    if (out_lo == out || (const float*)out == p_hi || (const float*)out == vt_hi || (p_lo && (const float*)out == p_lo) ||
        (vt_lo && (const float*)out == vt_lo))
        return set_error(GBX_EINVAL, "gbx_attn_values: out aliases an operand");
    const HeadsOperand x{p_hi, p_lo, S, (int64_t)S * S, (int64_t)H * S * S, S, false};
    const HeadsOperand w{vt_hi, vt_lo, S, (int64_t)hd * S, (int64_t)H * hd * S, hd, false};
    return heads_gemm("gbx_attn_values", x, w, out, out_lo, ld_out, hd, (int64_t)S * ld_out, B, H, S, hd, S, 0,
                      causal ? 1 : 0, err_flag, reinterpret_cast<cudaStream_t>(stream), 32);
}

extern "C" int gbx_transpose_heads(const float* v, int64_t ld, float* vt, int B, int S, int H, int hd,
                                   gbx_stream_t stream)
{
    if (int rc = heads_dims("gbx_transpose_heads", B, S, H, hd)) return rc;
    if (ld < (int64_t)H * hd) return set_error(GBX_EINVAL, "gbx_transpose_heads: ld=%lld < H*hd", (long long)ld);
    if (!v || !vt) return set_error(GBX_EINVAL, "gbx_transpose_heads: null pointer");
    if ((const float*)vt == v) return set_error(GBX_EINVAL, "gbx_transpose_heads: vt aliases v");
    const dim3 grid((unsigned)((S + 31) / 32), (unsigned)((hd + 31) / 32), (unsigned)(B * H));
    if (grid.y > 65535) return set_error(GBX_ERANGE, "gbx_transpose_heads: hd=%d", hd);
    transpose_heads_kernel<<<grid, dim3(32, 8), 0, reinterpret_cast<cudaStream_t>(stream)>>>(v, ld, vt, S, H, hd);
    return check_launch("gbx_transpose_heads");
}

// ------------------------------------------------------------------ split K
// y[m, n] = act(sum_s ws[s][m][n] + bias[n]) + resid[m, n], the slices added
// in the order s = 0, 1, ... (so results do not depend on scheduling), then
// the tf32 split when y_lo is given: gbx_linear's epilogue on the summed
// K slices.
template <bool VEC>
__global__ void __launch_bounds__(256)
splitk_reduce_kernel(const float* __restrict__ ws, int ksplit, const LinearArgs a)
{
    const int64_t MN = a.M * (int64_t)a.N;
    if constexpr (VEC) {
        const int64_t n4 = MN / 4;
        for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
             i += (int64_t)gridDim.x * blockDim.x) {
            float4 v = *reinterpret_cast<const float4*>(ws + 4 * i);
            for (int s = 1; s < ksplit; ++s) {
                const float4 w = *reinterpret_cast<const float4*>(ws + s * MN + 4 * i);
                v = add4(v, w);
            }
            // the epilogue of epi_store16, on 4 columns (N % 4 == 0: all in one row)
            const int n = (int)((4 * i) % a.N);
            if (a.bias) v = add4(v, __ldg(reinterpret_cast<const float4*>(a.bias + n)));
            if (a.act == GBX_ACT_GELU) v = gelu4(v);
            if (a.resid) v = add4(*reinterpret_cast<const float4*>(a.resid + 4 * i), v);
            if (a.y_lo) {
                float4 h, l;
                split4(v, h, l);
                *reinterpret_cast<float4*>(a.y + 4 * i) = h;
                *reinterpret_cast<float4*>(a.y_lo + 4 * i) = l;
            } else {
                *reinterpret_cast<float4*>(a.y + 4 * i) = v;
            }
        }
    } else {
        for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < MN; i += (int64_t)gridDim.x * blockDim.x) {
            float v = ws[i];
            for (int s = 1; s < ksplit; ++s) v += ws[s * MN + i];
            const int64_t row = i / a.N;
            const int n = (int)(i - row * a.N);
            const float o = epi_value(v, n, row, a);
            if (a.y_lo) {
                float h, l;
                split_value(o, h, l);
                a.y[i] = h;
                a.y_lo[i] = l;
            } else {
                a.y[i] = o;
            }
        }
    }
}

// gbx_linear with K cut into ksplit slices of K / ksplit: every slice is a
// "head" of the heads mode (its x and w columns a box offset in K), written
// as fp32 partial sums into ws, then splitk_reduce_kernel adds the slices and
// applies the epilogue.  Returns GBX_OK after enqueueing both launches.
static int linear_splitk(const float* x_hi, const float* x_lo, const float* w_hi, const float* w_lo, const float* bias,
                         const float* resid, float* y, float* y_lo, int64_t M, int N, int K, int act, int ksplit,
                         float* ws, int* err_flag, cudaStream_t s, const char* what)
{
    const int Kp = K / ksplit;
    const HeadsOperand x{x_hi, x_lo, K, Kp, 0, (int)M, true};
    const HeadsOperand w{w_hi, w_lo, K, Kp, 0, N, true};
    int rc = heads_gemm(what, x, w, ws, nullptr, N, M * (int64_t)N, 0, 1, ksplit, (int)M, N, Kp, 0, 0, err_flag, s);
    if (rc != GBX_OK) return rc;
    LinearArgs a;
    a.bias = bias;
    a.resid = resid;
    a.y = y;
    a.y_lo = y_lo;
    a.err = err_flag;
    a.M = M;
    a.N = N;
    a.K = K;
    a.act = act;
    const bool vec = N % 4 == 0 && aligned16(y) && (!y_lo || aligned16(y_lo)) && (!resid || aligned16(resid)) &&
                     (!bias || aligned16(bias)) && aligned16(ws);
    const int64_t work = vec ? (M * (int64_t)N / 4 + 255) / 256 : (M * (int64_t)N + 255) / 256;
    if (vec) {
        const int grid = persistent_grid(splitk_reduce_kernel<true>, 256, 0, work, 8);
        if (grid < 1) return GBX_ECUDA;
        splitk_reduce_kernel<true><<<grid, 256, 0, s>>>(ws, ksplit, a);
    } else {
        const int grid = persistent_grid(splitk_reduce_kernel<false>, 256, 0, work, 8);
        if (grid < 1) return GBX_ECUDA;
        splitk_reduce_kernel<false><<<grid, 256, 0, s>>>(ws, ksplit, a);
    }
    return check_launch(what);
}

// Arguments of the split-K entry points: GBX_OK, or the code gbx_linear
// would return; *use_split is false when the call should simply run
// gbx_linear (ksplit 1, or a shape the sliced tensor maps cannot take).
static int splitk_args(const char* what, const float* x_hi, const float* x_lo, const float* w_hi, const float* w_lo,
                       const float* y, const float* y_lo, int64_t M, int N, int K, int ksplit, bool* use_split)
{
    *use_split = false;
    if (ksplit < 1 || ksplit > kLinMaxSplit) return set_error(GBX_EINVAL, "%s: ksplit=%d", what, ksplit);
    if (M < 0 || N <= 0 || K <= 0) return set_error(GBX_EINVAL, "%s: M=%lld N=%d K=%d", what, (long long)M, N, K);
    if (M > 0x7fffffffLL) return set_error(GBX_ERANGE, "%s: M=%lld", what, (long long)M);
    auto al16 = [](const void* p) { return p == nullptr || aligned16(p); };
    *use_split = ksplit > 1 && M > 0 && K % ksplit == 0 && (K / ksplit) % 4 == 0 && x_hi && w_hi && y &&
                 al16(x_hi) && al16(x_lo) && al16(w_hi) && al16(w_lo) && y_lo != y;
    return GBX_OK;
}

extern "C" int gbx_linear_splitk(const float* x_hi, const float* x_lo, const float* w_hi, const float* w_lo,
                                 const float* bias, const float* resid, float* y, float* y_lo, int64_t M, int N, int K,
                                 int act, int ksplit, float* workspace, int64_t workspace_floats, int* err_flag,
                                 gbx_stream_t stream)
{
    bool split = false;
    if (int rc = splitk_args("gbx_linear_splitk", x_hi, x_lo, w_hi, w_lo, y, y_lo, M, N, K, ksplit, &split)) return rc;
    if (!split) return gbx_linear(x_hi, x_lo, w_hi, w_lo, bias, resid, y, y_lo, M, N, K, act, err_flag, stream);
    if (act != GBX_ACT_NONE && act != GBX_ACT_GELU) return set_error(GBX_EINVAL, "gbx_linear_splitk: act=%d", act);
    if (!workspace || workspace_floats < (int64_t)ksplit * M * N)
        return set_error(GBX_EINVAL, "gbx_linear_splitk: workspace of %lld floats, %lld needed",
                         (long long)workspace_floats, (long long)ksplit * M * N);
    const float* ws_end = workspace + (int64_t)ksplit * M * N;
    auto overlaps = [&](const float* p, int64_t n) { return p && p < ws_end && workspace < p + n; };
    if (overlaps(y, M * (int64_t)N) || overlaps(y_lo, M * (int64_t)N) || overlaps(resid, M * (int64_t)N) ||
        overlaps(x_hi, M * (int64_t)K) || overlaps(x_lo, M * (int64_t)K) || overlaps(w_hi, (int64_t)N * K) ||
        overlaps(w_lo, (int64_t)N * K))
        return set_error(GBX_EINVAL, "gbx_linear_splitk: workspace overlaps an operand");
    return linear_splitk(x_hi, x_lo, w_hi, w_lo, bias, resid, y, y_lo, M, N, K, act, ksplit, workspace, err_flag,
                         reinterpret_cast<cudaStream_t>(stream), "gbx_linear_splitk");
}

// ------------------------------------------------------------------ split K, no allocation
// gbx_linear_splitk for callers that cannot allocate device memory: the
// partial sums go to this file-scope array instead of a caller's workspace.
// Every GPU that loads the library holds it (16 MiB) until the process exits.
// Its name is only a host-side stand-in in host code; the device address
// comes from cudaGetSymbolAddress, once per device (splitk_scratch_of).
constexpr int64_t kNoAllocScratchFloats = (int64_t)1 << 22;
static __device__ __align__(256) float g_splitk_scratch[kNoAllocScratchFloats];

// The scratch array's device address on the current device, looked up on
// the first call for that device (with it current) and cached; nullptr and a
// recorded error when the runtime cannot give it.
static float* splitk_scratch_of(const char* what)
{
    constexpr int kMaxDevices = 64;
    static std::mutex mu;
    static float* addr[kMaxDevices] = {};
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        set_error(GBX_ECUDA, "%s: no current CUDA device (or device %d beyond %d)", what, dev, kMaxDevices);
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_splitk_scratch);
        if (e != cudaSuccess || !p) {
            set_error(GBX_ECUDA, "%s: cudaGetSymbolAddress of the scratch array failed: %s", what, cudaGetErrorString(e));
            return nullptr;
        }
        addr[dev] = static_cast<float*>(p);
    }
    return addr[dev];
}

extern "C" int gbx_linear_splitk_noalloc(const float* x_hi, const float* x_lo, const float* w_hi, const float* w_lo,
                                         const float* bias, const float* resid, float* y, float* y_lo, int64_t M, int N,
                                         int K, int act, int ksplit, int* err_flag, gbx_stream_t stream)
{
    bool split = false;
    if (int rc = splitk_args("gbx_linear_splitk_noalloc", x_hi, x_lo, w_hi, w_lo, y, y_lo, M, N, K, ksplit, &split))
        return rc;
    if (!split) return gbx_linear(x_hi, x_lo, w_hi, w_lo, bias, resid, y, y_lo, M, N, K, act, err_flag, stream);
    if (act != GBX_ACT_NONE && act != GBX_ACT_GELU)
        return set_error(GBX_EINVAL, "gbx_linear_splitk_noalloc: act=%d", act);
    if ((int64_t)ksplit * M * N > kNoAllocScratchFloats)
        return set_error(GBX_ERANGE,
                         "gbx_linear_splitk_noalloc: ksplit * M * N = %lld partial sums exceed the library's scratch "
                         "of %lld floats; use gbx_linear_splitk with a workspace",
                         (long long)ksplit * M * N, (long long)kNoAllocScratchFloats);
    float* ws = splitk_scratch_of("gbx_linear_splitk_noalloc");
    if (!ws) return GBX_ECUDA;
    return linear_splitk(x_hi, x_lo, w_hi, w_lo, bias, resid, y, y_lo, M, N, K, act, ksplit, ws, err_flag,
                         reinterpret_cast<cudaStream_t>(stream), "gbx_linear_splitk_noalloc");
}
