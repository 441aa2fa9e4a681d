// attention.cu -- causal self-attention of every head of every sequence in
// one kernel on the sm_100a tensor cores, replacing attentionScoresKernel,
// the per-head softmaxKernel launches and attentionOutputKernel
// (transformer.cu:213-249, launched at :834-846):
//   out[b, p, h*64 + i] = sum_s softmax_s(q_p . k_s / scale, s <= p) v[s, i]
// without the [S, S] scores or probabilities ever reaching HBM.
//
// Precision is that of the rest of the library: every operand is a tf32 pair
// and each product is formed as hi.hi + hi.lo + lo.hi; TMEM accumulates at
// most 64 products of a sum (one head width, or one step of 64 keys), and
// the output is summed over the steps in fp32 registers.  The softmax is the
// online form: per row a running maximum m and sum l of the raw scores x,
// weights e = 2^(x c - m c) with c = log2(e) / scale (one FFMA and the
// hardware's base-2 exponential), and a rescale of the running output by
// 2^((m_old - m_new) c) when the maximum grows; keys past the diagonal weigh
// exactly 0 and the output is divided by l exactly.  It differs from the
// reference's single-pass softmax only in rounding (about 2^-21 of each
// weight: the exponential's approximation and the rounding of x c; the
// weights' tf32 pair carries them to 2^-21 as well).
//
// One CTA works on one (head, 128-query tile) unit at a time, persistent over
// the units (longest first, each round of units dealt in the opposite
// direction to the last), 352 threads:
//   warp 0      TMA producer: the unit's Q tile (128 x 64, hi and lo), then per
//               step of 64 keys the K tile and the V tile into a two-stage
//               ring (128-byte swizzled rows, 32 floats per block), both
//               straight from the QKV rows: V is the MMA's B operand in
//               MN-major form (head columns contiguous, 32-byte swizzle
//               atoms, the one layout of an MN-major tf32 operand), so no
//               transpose
//   warp 1      owns 512 TMEM columns; one thread issues the score MMAs
//                 S[j] = Q K_j^T                      (kind::tf32, M 128, N 64)
//   warp 2      one thread issues the value MMAs
//                 O[j] = P_j V_j                      (A = P_j from TMEM)
//               (at N 64, 24 MMAs per product and step, one thread issuing
//               both bounded the kernel); S[j+1] runs while the softmax
//               warps work on S[j]
//   warps 3-10  softmax: warps w and w + 4 own query rows 32 (w % 4) .. +31,
//               32 of the 64 columns each; a thread reads its S[j] columns
//               from TMEM, writes its part of P_j as a tf32 pair back into
//               TMEM (hi over S[j]), then adds its 32 columns of O[j-1] into
//               fp32 registers with the pending rescale.  A unit's last
//               output and its rows wait until the next unit's first P is
//               written; each warp's 32 x 32 block of rows leaves through a
//               shared-memory staging block (64 contiguous bytes of 8 rows a
//               store instruction)
// TMEM columns: S/P_hi [0,64) and [64,128), P_lo [128,192) and [192,256),
// O [256,320) and [320,384), each double-buffered by step parity.
// Every mbarrier wait is bounded (1 s, %globaltimer): a wait that runs out
// sets the CTA's abort word, every role leaves its loops, loads and MMAs in
// flight are waited for (bounded), TMEM is freed and GBX_LINEAR_TIMEOUT is
// OR-ed into the error flag.  No cluster multicast.
#include <cuda.h>

#include "gbx_common.cuh"
#include "tcgen05.cuh"
#include "tensormap.cuh"
#include "tf32.cuh"

namespace gbx {

constexpr int kAttQ = 128;        // query rows per unit (TMEM lanes)
constexpr int kAttKT = 64;        // keys per step
constexpr int kAttHD = 64;        // head width
constexpr int kAttSoftWarps = 8;
constexpr int kAttThreads = 96 + 32 * kAttSoftWarps;
constexpr uint64_t kAttWaitNs = 1000000000ull;
// shared memory: Q (2 planes x 2 K blocks x 128 rows x 128 B), then two ring
// stages of K (2 x 2 x 64 rows x 128 B) and V (the same)
constexpr uint32_t kAttQBlock = 128 * 128;                 // one plane, one K block of Q
constexpr uint32_t kAttKVBlock = 64 * 128;                 // one plane, 32 columns of K or V
constexpr uint32_t kAttQBytes = 4 * kAttQBlock;            // 64 KB
constexpr uint32_t kAttKVBytes = 4 * kAttKVBlock;          // 32 KB
constexpr uint32_t kAttStages = 2;
constexpr uint32_t kAttData = kAttQBytes + kAttStages * 2 * kAttKVBytes;   // 192 KB
// barriers: qfull qempty kfull[2] kempty[2] vfull[2] vempty[2] sfull[2] pfull[2] pvdone[2] ofull[2] oempty[2]
// drain drain2
constexpr int kAttBars = 22;
// after the barriers and the TMEM slot: the softmax halves' exchange slots
constexpr size_t kAttXBytes = 2 * 4 * 2 * 32 * sizeof(float);
// then each softmax warp's output staging block: 32 rows x 16 floats
constexpr size_t kAttStageBytes = kAttSoftWarps * 32 * 16 * sizeof(float);
constexpr size_t kAttSmem = kAttData + 1024 + 8 * kAttBars + 16 + kAttXBytes + kAttStageBytes;
constexpr uint32_t kTmS = 0, kTmPlo = 128, kTmO = 256, kTmCols = 512;

struct AttnArgs {
    float* out;
    float* out_lo;
    int64_t ld_out;
    int B, S, H;
    int nqt;      // query tiles per head
    int units;    // B * H * nqt
    float c2;     // log2(e) / scale: a weight is 2^(x c2 - m c2) for raw score x, row maximum m
    int causal;
    int* err;
};

struct AttnUnit {
    int b, h, qt, nkt;
};

__device__ __forceinline__ AttnUnit attn_unit(int u, const AttnArgs& a)
{
    const int Z = a.B * a.H;
    AttnUnit w;
    w.qt = a.nqt - 1 - u / Z;   // the longest query tiles first
    const int z = u - (u / Z) * Z;
    w.b = z / a.H;
    w.h = z - w.b * a.H;
    const int kend = a.causal ? min(a.S, (w.qt + 1) * kAttQ) : a.S;
    w.nkt = (kend + kAttKT - 1) / kAttKT;
    return w;
}

// The unit a CTA takes in its k-th round (a.units when none is left):
// rounds of gridDim.x units in the longest-first order, dealt forwards in
// even rounds and backwards in odd ones, so a CTA that drew a longer unit
// in one round draws a shorter one in the next.  For 8 x 16 heads x 1024
// causal on 148 SMs the busiest CTA gets 64 key steps (70 dealt forwards
// every round; 62.3 on average); for one sequence of 25 heads, 16 (22).
__device__ __forceinline__ int attn_round_unit(int k, const AttnArgs& a)
{
    const long long G = gridDim.x;
    const long long u = k * G + ((k & 1) ? G - 1 - (long long)blockIdx.x : (long long)blockIdx.x);
    return u < a.units ? (int)u : a.units;
}

// 2^x by the hardware's base-2 approximation (ex2.approx, subnormal results
// flushed to 0: such a weight is below 2^-126 of the row's largest, which
// weighs 1).  The softmax's exponentials are e^y = 2^(y log2 e), with the
// 1/scale folded into the same constant.
__device__ __forceinline__ float att_exp2(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float att_div(float x, float d, float rd)
{
    const float q = x * rd;
    return fmaf(fmaf(-q, d, x), rd, q);
}

__global__ void __launch_bounds__(kAttThreads, 1)
attn_fused_kernel(const __grid_constant__ CUtensorMap map_qh, const __grid_constant__ CUtensorMap map_ql,
                  const __grid_constant__ CUtensorMap map_kh, const __grid_constant__ CUtensorMap map_kl,
                  const __grid_constant__ CUtensorMap map_vh, const __grid_constant__ CUtensorMap map_vl,
                  const AttnArgs a)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kAttData);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kAttBars);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const uint32_t b0 = tc::smem_u32(bars);
    const uint32_t qfull = b0, qempty = b0 + 8;
    auto kfull = [&](int s) { return b0 + 16 + 8 * s; };
    auto kempty = [&](int s) { return b0 + 32 + 8 * s; };
    auto vfull = [&](int s) { return b0 + 48 + 8 * s; };
    auto vempty = [&](int s) { return b0 + 64 + 8 * s; };
    auto sfull = [&](int i) { return b0 + 80 + 8 * i; };
    auto pfull = [&](int i) { return b0 + 96 + 8 * i; };
    auto pvdone = [&](int i) { return b0 + 112 + 8 * i; };
    auto ofull = [&](int i) { return b0 + 128 + 8 * i; };
    auto oempty = [&](int i) { return b0 + 144 + 8 * i; };
    const uint32_t drain = b0 + 160, drain2 = b0 + 168;
    const uint32_t smem0 = tc::smem_u32(smem);
    const uint32_t qbase = smem0;
    auto kbase = [&](int s) { return smem0 + kAttQBytes + s * 2 * kAttKVBytes; };
    auto vbase = [&](int s) { return smem0 + kAttQBytes + s * 2 * kAttKVBytes + kAttKVBytes; };

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        tc::mbar_init(qfull, 1);
        tc::mbar_init(qempty, 1);
        for (int s = 0; s < 2; ++s) {
            tc::mbar_init(kfull(s), 1);
            tc::mbar_init(kempty(s), 1);
            tc::mbar_init(vfull(s), 1);
            tc::mbar_init(vempty(s), 1);
            tc::mbar_init(sfull(s), 1);
            tc::mbar_init(pfull(s), kAttSoftWarps);
            tc::mbar_init(pvdone(s), 1);
            tc::mbar_init(ofull(s), 1);
            tc::mbar_init(oempty(s), kAttSoftWarps);
        }
        tc::mbar_init(drain, 1);
        tc::mbar_init(drain2, 1);
        *abort = 0;
        tc::fence_mbar_init();
        tc::tma_prefetch(&map_qh);
        tc::tma_prefetch(&map_ql);
        tc::tma_prefetch(&map_kh);
        tc::tma_prefetch(&map_kl);
        tc::tma_prefetch(&map_vh);
        tc::tma_prefetch(&map_vl);
    }
    if (warp == 1) {
        tc::tmem_alloc(tc::smem_u32(tmem_slot), kTmCols);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------------------------------------------- producer
            int st = 0;
            uint32_t ph = 0, qph = 0;
            bool ok = true;
            int q_loads = 0;
            uint32_t issued = 0, lastpar = 0;   // ring stages with loads issued, parity of their last phase
            for (int k = 0, u = attn_round_unit(0, a); u < a.units && ok; u = attn_round_unit(++k, a)) {
                const AttnUnit w = attn_unit(u, a);
                if (!tc::mbar_wait(qempty, qph ^ 1, abort, kAttWaitNs)) break;
                tc::mbar_arrive_expect_tx(qfull, kAttQBytes);
                for (int p = 0; p < 2; ++p)
                    for (int kb = 0; kb < 2; ++kb)
                        tc::tma_load_4d(qbase + (2 * p + kb) * kAttQBlock, p ? &map_ql : &map_qh, qfull, 32 * kb, w.h,
                                        w.qt * kAttQ, w.b);
                ++q_loads;
                qph ^= 1;
                for (int j = 0; j < w.nkt; ++j) {
                    if (!tc::mbar_wait(kempty(st), ph ^ 1, abort, kAttWaitNs)) {
                        ok = false;
                        break;
                    }
                    tc::mbar_arrive_expect_tx(kfull(st), kAttKVBytes);
                    for (int p = 0; p < 2; ++p)
                        for (int kb = 0; kb < 2; ++kb)
                            tc::tma_load_4d(kbase(st) + (2 * p + kb) * kAttKVBlock, p ? &map_kl : &map_kh, kfull(st),
                                            32 * kb, w.h, j * kAttKT, w.b);
                    if (!tc::mbar_wait(vempty(st), ph ^ 1, abort, kAttWaitNs)) {
                        ok = false;
                        break;
                    }
                    tc::mbar_arrive_expect_tx(vfull(st), kAttKVBytes);
                    for (int p = 0; p < 2; ++p)
                        for (int kb = 0; kb < 2; ++kb)
                            tc::tma_load_4d(vbase(st) + (2 * p + kb) * kAttKVBlock, p ? &map_vl : &map_vh, vfull(st),
                                            32 * kb, w.h, j * kAttKT, w.b);
                    issued |= 1u << st;
                    lastpar = (lastpar & ~(1u << st)) | (ph << st);
                    if (++st == 2) {
                        st = 0;
                        ph ^= 1;
                    }
                }
            }
            // every load issued has landed before the CTA may exit
            if (q_loads) tc::mbar_wait(qfull, (q_loads - 1) & 1, nullptr, kAttWaitNs);
            for (int s = 0; s < 2; ++s)
                if (issued & (1u << s)) {
                    tc::mbar_wait(kfull(s), (lastpar >> s) & 1, nullptr, kAttWaitNs);
                    tc::mbar_wait(vfull(s), (lastpar >> s) & 1, nullptr, kAttWaitNs);
                }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------------------------------------- score MMA issuer
            const uint32_t idesc = tc::idesc_tf32(kAttQ, kAttKT);   // M 128, N 64
            // shared-memory descriptors of the K blocks' first K step; a K
            // step of 8 floats advances the address field by 32 bytes
            const uint64_t dq = tc::smem_desc(qbase, 128);
            int kst = 0;
            uint32_t kph = 0, qph = 0;
            uint32_t g = 0;   // global step (buffer = g & 1, its use count = g >> 1)
            bool ok = true;
            for (int k = 0, u = attn_round_unit(0, a); u < a.units && ok; u = attn_round_unit(++k, a)) {
                const AttnUnit w = attn_unit(u, a);
                if (!tc::mbar_wait(qfull, qph, abort, kAttWaitNs)) break;
                qph ^= 1;
                for (int j = 0; j < w.nkt; ++j, ++g) {
                    const uint32_t i = g & 1;
                    // S[g] overwrites buffer i: P_{g-2} there has been read by its MMA
                    if (g >= 2 && !tc::mbar_wait(pvdone(i), ((g - 2) >> 1) & 1, abort, kAttWaitNs)) {
                        ok = false;
                        break;
                    }
                    if (!tc::mbar_wait(kfull(kst), kph, abort, kAttWaitNs)) {
                        ok = false;
                        break;
                    }
                    tc::fence_after_sync();
                    const uint32_t d = tmem + kTmS + 64 * i;
                    const uint64_t dk = tc::smem_desc(kbase(kst), 128);
#pragma unroll
                    for (int kb = 0; kb < 2; ++kb)
#pragma unroll
                        for (int ks = 0; ks < 4; ++ks) {
                            const uint64_t qh = dq + ((kb * kAttQBlock + 32 * ks) >> 4);
                            const uint64_t ql = dq + (((2 + kb) * kAttQBlock + 32 * ks) >> 4);
                            const uint64_t kh = dk + ((kb * kAttKVBlock + 32 * ks) >> 4);
                            const uint64_t kl = dk + (((2 + kb) * kAttKVBlock + 32 * ks) >> 4);
                            tc::mma_tf32(d, qh, kh, idesc, (kb | ks) != 0);
                            tc::mma_tf32(d, qh, kl, idesc, 1);
                            tc::mma_tf32(d, ql, kh, idesc, 1);
                        }
                    tc::mma_commit(sfull(i));
                    tc::mma_commit(kempty(kst));
                    if (j == w.nkt - 1) tc::mma_commit(qempty);   // the unit's last read of Q
                    if (++kst == 2) {
                        kst = 0;
                        kph ^= 1;
                    }
                }
            }
            // every MMA this thread issued has completed before TMEM is freed
            tc::mma_commit(drain);
            tc::mbar_wait(drain, 0, nullptr, kAttWaitNs);
        }
    } else if (warp == 2) {
        if (lane == 0) {
            // --------------------------------------------- values MMA issuer
            // O[g] = P_g V_g with P_g read from TMEM.  A second issuing thread:
            // at N 64 one thread issuing both products bounds the kernel.
            const uint32_t idesc = tc::idesc_tf32_bmn(kAttQ, kAttHD);   // M 128, N 64, B MN-major
            int vst = 0;
            uint32_t vph = 0;
            uint32_t g = 0;
            bool ok = true;
            for (int k = 0, u = attn_round_unit(0, a); u < a.units && ok; u = attn_round_unit(++k, a)) {
                const AttnUnit w = attn_unit(u, a);
                for (int j = 0; j < w.nkt; ++j, ++g) {
                    const uint32_t i = g & 1;
                    if (!tc::mbar_wait(pfull(i), (g >> 1) & 1, abort, kAttWaitNs) ||
                        !tc::mbar_wait(vfull(vst), vph, abort, kAttWaitNs) ||
                        (g >= 2 && !tc::mbar_wait(oempty(i), ((g - 2) >> 1) & 1, abort, kAttWaitNs))) {
                        ok = false;
                        break;
                    }
                    tc::fence_after_sync();
                    const uint32_t d = tmem + kTmO + 64 * i;
                    const uint32_t phi = tmem + kTmS + 64 * i, plo = tmem + kTmPlo + 64 * i;
                    // V is MN-major: key rows of 128 bytes (32 head columns) in
                    // 4-row (512 B) swizzle atoms, a K step of 8 keys is 1 KB,
                    // head columns 32..63 sit one box (8 KB) on, the low plane
                    // two boxes on
                    const uint64_t dv = tc::smem_desc_mn128_b32(vbase(vst), kAttKVBlock, 512);
#pragma unroll
                    for (int t = 0; t < kAttKT / 8; ++t) {
                        const uint32_t k8 = 8 * t;   // key column of this K step
                        const uint64_t vh = dv + ((1024u * t) >> 4);
                        const uint64_t vl = dv + ((2 * kAttKVBlock + 1024u * t) >> 4);
                        tc::mma_tf32_ts(d, phi + k8, vh, idesc, t != 0);
                        tc::mma_tf32_ts(d, phi + k8, vl, idesc, 1);
                        tc::mma_tf32_ts(d, plo + k8, vh, idesc, 1);
                    }
                    tc::mma_commit(ofull(i));
                    tc::mma_commit(vempty(vst));
                    tc::mma_commit(pvdone(i));
                    if (++vst == 2) {
                        vst = 0;
                        vph ^= 1;
                    }
                }
            }
            tc::mma_commit(drain2);
            tc::mbar_wait(drain2, 0, nullptr, kAttWaitNs);
        }
    } else {
        // -------------------------------------------------------- softmax
        // Warps w and w + 4 (3 <= w <= 6) share query rows 32 (w % 4) .. +31 (the TMEM lane
        // quarter they may read); `half` picks the 32 of the 64 key (and
        // output) columns this thread owns.  The two halves of a row exchange
        // their step maxima through shared memory (double-buffered by step
        // parity) at a 64-thread named barrier, keep their own partial sums
        // (the same rescales apply to both) and add them at the end.
        const int quarter = warp & 3;
        const int half = (warp - 3) >> 2;
        const int row_in_tile = 32 * quarter + lane;
        const uint32_t lane_addr = (uint32_t)(32 * quarter) << 16;
        const uint32_t col = 32 * half;
        float* const xmax = reinterpret_cast<float*>(tmem_slot + 4);   // [2 parity][4 quarter][2 half][32]
        float* const stage = xmax + 2 * 4 * 2 * 32 + (warp - 3) * 32 * 16;
        const int bar_id = 1 + quarter;                             // named barriers 1-4
        // The pair's barrier also decides, for both halves alike, whether to
        // stop: it returns the OR of the two halves' `stop` (a half never
        // leaves its loop alone, which would leave the other waiting at the
        // barrier for ever).
        auto pair_sync = [&](bool stop) -> bool {
            uint32_t any;
            asm volatile(
                "{\n\t.reg .pred p, q;\n\t"
                "setp.ne.u32 q, %2, 0;\n\t"
                "bar.red.or.pred p, %1, 64, q;\n\t"
                "selp.u32 %0, 1, 0, p;\n\t}"
                : "=r"(any)
                : "r"(bar_id), "r"((uint32_t)stop)
                : "memory");
            return any != 0;
        };
        uint32_t g = 0;
        bool ok = true;
        float o[32];   // the running output of this thread's 32 columns
#pragma unroll
        for (int c = 0; c < 32; ++c) o[c] = 0.0f;
        float alpha_pend = 0.0f;
        // adds O[gg] (the running output rescaled first) and releases its buffer
        auto take_o = [&](uint32_t gg, float alpha) -> bool {
            const uint32_t i = gg & 1;
            const bool ready = tc::mbar_wait(ofull(i), (gg >> 1) & 1, abort, kAttWaitNs);
            if (!__all_sync(0xffffffffu, ready)) return false;
            tc::fence_after_sync();
            float v[32];
            tc::tmem_ld32(tmem + lane_addr + kTmO + 64 * i + col, v);
            tc::tmem_ld_wait();
#pragma unroll
            for (int c = 0; c < 32; ++c) o[c] = fmaf(o[c], alpha, v[c]);
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(oempty(i));
            return true;
        };
        // A unit's last output and its epilogue (the two halves' row sums
        // added, the division, the stores) wait until the next unit's first
        // step has written its P: the tensor pipe runs that step's value
        // product and the next score product meanwhile, instead of waiting
        // for the epilogue.  `pend`: unit pw (this half's row sum pl) waits.
        bool pend = false;
        AttnUnit pw{};
        float pl = 0.0f;
        // Takes pw's last output O[g - 1], writes pw's rows and clears the
        // running output; false stops both halves (decided at the pair's
        // barrier).  xpar: the exchange slot's parity, one that no half
        // reads any more (not that of the step whose barrier was passed last).
        auto finish = [&](bool good, uint32_t xpar) -> bool {
            good = good && take_o(g - 1, alpha_pend);
            float* const xl = xmax + (((xpar * 4 + quarter) * 2) * 32);
            xl[half * 32 + lane] = pl;
            if (pair_sync(!good)) return false;
            const float lsum = pl + xl[(1 - half) * 32 + lane];
            pair_sync(false);   // the slot is read before either half writes it again
            {
                const float rl = 1.0f / lsum;
#pragma unroll
                for (int c = 0; c < 32; ++c) o[c] = att_div(o[c], lsum, rl);
            }
            // The warp's 32 rows x 32 columns leave through its staging block,
            // 16 columns of one plane at a time: each lane writes 64 bytes of
            // its own row, then each store instruction writes 64 contiguous
            // bytes of 8 rows (a lane per 16 bytes) instead of 16 bytes of 32
            // rows.  16-byte chunk c of row r sits at chunk c ^ ((r >> 1) & 3)
            // (conflict-free both ways).
            {
                const int r0 = pw.qt * kAttQ + 32 * quarter;   // the warp's first query row
                const int64_t base = ((int64_t)pw.b * a.S + r0) * a.ld_out + (int64_t)pw.h * kAttHD + col;
                const int rr = lane >> 2, cq = lane & 3;          // read side: row in an 8-row group, chunk
#pragma unroll
                for (int pn = 0; pn < 2; ++pn) {
                    if (pn == 1 && !a.out_lo) break;
                    float* const dst = pn ? a.out_lo : a.out;
#pragma unroll
                    for (int hb = 0; hb < 2; ++hb) {
                        __syncwarp();
#pragma unroll
                        for (int cc = 0; cc < 4; ++cc) {
                            float4 v = make_float4(o[16 * hb + 4 * cc], o[16 * hb + 4 * cc + 1], o[16 * hb + 4 * cc + 2],
                                                   o[16 * hb + 4 * cc + 3]);
                            if (a.out_lo) {
                                float4 h4, l4;
                                split4(v, h4, l4);
                                v = pn ? l4 : h4;
                            }
                            *reinterpret_cast<float4*>(stage + lane * 16 + 4 * (cc ^ ((lane >> 1) & 3))) = v;
                        }
                        __syncwarp();
#pragma unroll
                        for (int t = 0; t < 4; ++t) {
                            const int r = 8 * t + rr;
                            const float4 v =
                                *reinterpret_cast<const float4*>(stage + r * 16 + 4 * (cq ^ ((r >> 1) & 3)));
                            if (r0 + r < a.S)
                                *reinterpret_cast<float4*>(dst + base + (int64_t)r * a.ld_out + 16 * hb + 4 * cq) = v;
                        }
                    }
                }
            }
#pragma unroll
            for (int c = 0; c < 32; ++c) o[c] = 0.0f;
            return true;
        };
        for (int k = 0, u = attn_round_unit(0, a); u < a.units; u = attn_round_unit(++k, a)) {
            const AttnUnit w = attn_unit(u, a);
            const int p = w.qt * kAttQ + row_in_tile;   // this thread's query position
            const int lim = a.causal ? min(p + 1, a.S) : a.S;
            float m = -INFINITY, l = 0.0f;
            bool broke = false;   // both halves left the step loop at the same barrier
            for (int j = 0; j < w.nkt; ++j, ++g) {
                const uint32_t i = g & 1;
                // a failed wait here or in the previous step's take_o stops
                // both halves at this step's barrier
                const bool ready =
                    ok && __all_sync(0xffffffffu, tc::mbar_wait(sfull(i), (g >> 1) & 1, abort, kAttWaitNs));
                float s[32];
                if (ready) {
                    tc::fence_after_sync();
                    tc::tmem_ld32(tmem + lane_addr + kTmS + 64 * i + col, s);
                    tc::tmem_ld_wait();
                } else {
#pragma unroll
                    for (int c = 0; c < 32; ++c) s[c] = 0.0f;
                }
                // keys k0 .. k0 + nvis - 1 of this thread's 32 are visible to its row
                const int k0 = j * kAttKT + (int)col;
                const int nvis = max(0, min(32, lim - k0));
                const bool full = __all_sync(0xffffffffu, nvis == 32);
                float mt = -INFINITY;   // on the raw scores (the maximum commutes with 1/scale)
                if (full) {
#pragma unroll
                    for (int c = 0; c < 32; ++c) mt = fmaxf(mt, s[c]);
                } else {
                    // hidden keys become -inf, whose weight 2^-inf is exactly 0
#pragma unroll
                    for (int c = 0; c < 32; ++c) {
                        s[c] = c < nvis ? s[c] : -INFINITY;
                        mt = fmaxf(mt, s[c]);
                    }
                }
                // the row's step maximum: both halves
                float* const xm = xmax + (((i * 4 + quarter) * 2) * 32);
                xm[half * 32 + lane] = mt;
                if (pair_sync(!ready)) {
                    broke = true;
                    break;
                }
                mt = fmaxf(mt, xm[(1 - half) * 32 + lane]);
                const float m_new = fmaxf(m, mt);
                // e^((x - m) / scale) = 2^(x c2 - m c2): one FFMA and one
                // exponential per weight (m_new is finite once a key is
                // visible; a hidden key's -inf gives 0).  One loop for full and
                // masked steps: two loops, one per case, spill at the
                // 168-register cap
                const float alpha = m_new == -INFINITY ? 1.0f : att_exp2((m - m_new) * a.c2);
                const float mc = m_new == -INFINITY ? 0.0f : m_new * a.c2;
                float sum = 0.0f;
#pragma unroll
                for (int c = 0; c < 32; ++c) {
                    s[c] = att_exp2(fmaf(s[c], a.c2, -mc));
                    sum += s[c];
                }
                l = fmaf(l, alpha, sum);
                m = m_new;
                // P as a tf32 pair, hi over S[g], lo in its own columns.  Each
                // weight is in [0, 1]: hi = the weight rounded to 10 mantissa
                // bits, ties away from 0 (carry 0x1000 into the kept bits,
                // clear the 13 dropped ones; two integer operations, where the
                // cvt.rna conversion measured slower), lo = the exact
                // remainder, whose own low 13 bits the MMA ignores (at most
                // 2^-21 of the weight)
                float lo[32];
#pragma unroll
                for (int c = 0; c < 32; ++c) {
                    const float h = __uint_as_float((__float_as_uint(s[c]) + 0x1000u) & 0xffffe000u);
                    lo[c] = s[c] - h;
                    s[c] = h;
                }
                tc::tmem_st32(tmem + lane_addr + kTmS + 64 * i + col, s);
                tc::tmem_st32(tmem + lane_addr + kTmPlo + 64 * i + col, lo);
                tc::tmem_st_wait();
                tc::fence_before_sync();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(pfull(i));
                if (j == 0) {
                    // the previous unit's last output and rows
                    if (pend && !finish(true, (g + 1) & 1)) {
                        broke = true;
                        break;
                    }
                    pend = false;
                } else if (!take_o(g - 1, alpha_pend)) {
                    ok = false;   // both stop at the next barrier (this unit's or the next's, or finish's)
                }
                alpha_pend = alpha;
            }
            if (broke) {
                ok = false;
                pend = false;
                break;
            }
            pend = true;
            pw = w;
            pl = l;
        }
        // the last unit (a failed take_o of its last step is decided here)
        if (pend && !finish(ok, g & 1)) ok = false;
    }

    __syncthreads();   // every role has left its loop (all waits are bounded)
    if (warp == 1) {
        __syncwarp();
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, kTmCols);
    }
    if (threadIdx.x == 0 && *abort && a.err) atomicOr(a.err, GBX_LINEAR_TIMEOUT);
}

// One plane of a heads-mode operand as a 4-D map: dims (inner k, then d1, d2,
// d3) with element strides s1 < s2 < s3, boxes of 32 x box1 x box2 x 1 and
// the 128-byte swizzle (16-byte atoms for the K-major Q and K; 32-byte atoms
// for V, the MMA's MN-major operand).
static int attn_map(CUtensorMap* m, const float* base, const cuuint64_t (&dims)[4], const cuuint64_t (&strides)[3],
                    cuuint32_t box1, cuuint32_t box2, CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B)
{
    EncodeTiledFn fn = encode_tiled();
    if (!fn) return set_error(GBX_ECUDA, "gbx_attn_fused: cuTensorMapEncodeTiled unavailable from the driver");
    cuuint64_t sb[3];
    for (int i = 0; i < 3; ++i) sb[i] = strides[i] * sizeof(float);
    const cuuint32_t box[4] = {32, box1, box2, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float*>(base), dims, sb, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(GBX_EINVAL, "gbx_attn_fused: tensor map rejected (CUresult %d)", (int)r);
    return GBX_OK;
}

}  // namespace gbx

using namespace gbx;

extern "C" int gbx_attn_fused(const float* q_hi, const float* q_lo, const float* k_hi, const float* k_lo, int64_t ld,
                              const float* v_hi, const float* v_lo, float* out, float* out_lo, int64_t ld_out, int B,
                              int S, int H, int hd, float scale, int causal, int* err_flag, gbx_stream_t stream)
{
    if (B <= 0 || S <= 0 || H <= 0 || hd <= 0)
        return set_error(GBX_EINVAL, "gbx_attn_fused: B=%d S=%d H=%d hd=%d", B, S, H, hd);
    if (hd != kAttHD) return set_error(GBX_EINVAL, "gbx_attn_fused: head width %d (64 only)", hd);
    if (!(scale >= 1.17549435e-38f) || scale == INFINITY)
        return set_error(GBX_EINVAL, "gbx_attn_fused: scale=%g must be a normal positive float", (double)scale);
    if (!q_hi || !q_lo || !k_hi || !k_lo || !v_hi || !v_lo || !out)
        return set_error(GBX_EINVAL, "gbx_attn_fused: null pointer");
    if (ld < (int64_t)H * hd || ld_out < (int64_t)H * hd)
        return set_error(GBX_EINVAL, "gbx_attn_fused: ld=%lld ld_out=%lld < H*hd", (long long)ld, (long long)ld_out);
    if (out_lo == out) return set_error(GBX_EINVAL, "gbx_attn_fused: out_lo aliases out");
    {
        // CTAs store their output rows while other CTAs still read Q, K and V:
        // no output may overlap an operand's extent
        const int64_t in_n = ((int64_t)B * S - 1) * ld + (int64_t)H * hd;
        const int64_t out_n = ((int64_t)B * S - 1) * ld_out + (int64_t)H * hd;
        auto overlaps = [](const float* a, int64_t na, const float* b, int64_t nb) {
            return a && b && b < a + na && a < b + nb;
        };
        for (const float* o : {(const float*)out, (const float*)out_lo})
            for (const float* in : {q_hi, q_lo, k_hi, k_lo, v_hi, v_lo})
                if (overlaps(o, out_n, in, in_n))
                    return set_error(GBX_EINVAL, "gbx_attn_fused: an output overlaps an operand");
        if (overlaps(out, out_n, out_lo, out_n)) return set_error(GBX_EINVAL, "gbx_attn_fused: out and out_lo overlap");
    }
    // the tensor maps: 16-byte bases and strides; the vector output stores
    const bool al = aligned16(q_hi) && aligned16(q_lo) && aligned16(k_hi) && aligned16(k_lo) && aligned16(v_hi) &&
                    aligned16(v_lo) && aligned16(out) && (!out_lo || aligned16(out_lo));
    if (!al || ld % 4 || ld_out % 4)
        return set_error(GBX_EINVAL, "gbx_attn_fused: operands need 16-byte alignment and ld, ld_out multiples of 4");
    const int nqt = (S + kAttQ - 1) / kAttQ;
    if ((int64_t)B * H * nqt > 0x7fffffffLL || (int64_t)B * S > 0x7fffffffLL)
        return set_error(GBX_ERANGE, "gbx_attn_fused: B=%d H=%d S=%d too large", B, H, S);
    DeviceInfo di;
    if (device_info(&di) != GBX_OK) return GBX_ECUDA;
    if ((size_t)di.max_smem_optin < kAttSmem)
        return set_error(GBX_ERANGE, "gbx_attn_fused: needs %zu bytes of shared memory per CTA", kAttSmem);

    // Q, K and V: element (b, s, h, i) at b*S*ld + s*ld + h*64 + i, dims (i, h, s, b)
    CUtensorMap mqh, mql, mkh, mkl, mvh, mvl;
    const cuuint64_t dqk[4] = {(cuuint64_t)hd, (cuuint64_t)H, (cuuint64_t)S, (cuuint64_t)B};
    const cuuint64_t sqk[3] = {(cuuint64_t)hd, (cuuint64_t)ld, (cuuint64_t)S * ld};
    int rc;
    if ((rc = attn_map(&mqh, q_hi, dqk, sqk, 1, kAttQ)) || (rc = attn_map(&mql, q_lo, dqk, sqk, 1, kAttQ)) ||
        (rc = attn_map(&mkh, k_hi, dqk, sqk, 1, kAttKT)) || (rc = attn_map(&mkl, k_lo, dqk, sqk, 1, kAttKT)) ||
        (rc = attn_map(&mvh, v_hi, dqk, sqk, 1, kAttKT, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B)) ||
        (rc = attn_map(&mvl, v_lo, dqk, sqk, 1, kAttKT, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B)))
        return rc;
    AttnArgs a;
    a.out = out;
    a.out_lo = out_lo;
    a.ld_out = ld_out;
    a.B = B;
    a.S = S;
    a.H = H;
    a.nqt = nqt;
    a.units = B * H * nqt;
    a.c2 = (float)(1.4426950408889634 / (double)scale);   // log2(e) / scale
    a.causal = causal ? 1 : 0;
    a.err = err_flag;
    if (cudaFuncSetAttribute(attn_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kAttSmem) !=
        cudaSuccess)
        return set_error(GBX_ECUDA, "gbx_attn_fused: shared-memory attribute refused");
    const int grid = a.units < di.sm_count ? a.units : di.sm_count;
    attn_fused_kernel<<<grid, kAttThreads, kAttSmem, reinterpret_cast<cudaStream_t>(stream)>>>(mqh, mql, mkh, mkl, mvh,
                                                                                              mvl, a);
    return check_launch("gbx_attn_fused");
}
