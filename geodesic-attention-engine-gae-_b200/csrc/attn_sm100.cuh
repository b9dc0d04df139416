// attn_sm100.cuh -- fused exact attention forward for B200 (sm_100a) on the
// 5th-generation tensor cores.
//
// Semantics: the reference's Waller operator (rust_src/src/waller_operator.rs
// :8-59): O[i] = sum_j softmax_j(scale * <Q_i, K_j>) V_j, one streaming pass
// over K/V with a running max and running sum per query row, no N x N
// intermediate.  The reference's GPU versions are cuda_src/waller_kernel_bench
// .cu:40-290 (cuBLAS tiles, S/P round-trip HBM) and cuda_src/bench_tma.cu:152-
// 429 (Hopper TMA + wgmma); this kernel is a new design for tcgen05/TMEM.
//
// Persistent CTAs (one per SM) walk a heaviest-first list of units; a unit is
// 256 query rows of one (batch, head): two 128-row Q tiles that ping-pong on
// the tensor core.  Warp roles (384 threads, 3 warpgroups):
//   warps 0-3  softmax group 0  (Q tile 0, TMEM lanes 0..127, thread = row)
//   warps 4-7  softmax group 1  (Q tile 1)
//   warp  8    TMA producer     (Q once, then K_j, V_j into a smem ring)
//   warp  9    MMA issuer       (owns the TMEM allocation)
//   warps 10-11 idle
// Registers: launched at 168 per thread; the producer warpgroup shrinks to
// 80 (96 in int8 mode) and the two softmax warpgroups grow to 208 (200):
// 2*128*208 + 128*80 and 2*128*200 + 128*96 are at most 384*168, so the
// re-balancing always fits.
// TMEM (512 columns): S0 [0,128), S1 [128,256), O0 [256,256+D), O1 after it.
// P_i (bf16, 2 per column) overwrites the first 64 columns of S_i and feeds
// the P*V MMA straight from TMEM.  Per K/V tile j the MMA warp issues
//   PV0(j-1), QK0(j), PV1(j-1), QK1(j)
// so S_i is rewritten only after the MMA that read P_i was issued (tcgen05
// MMAs of one thread execute in issue order), and the commit that publishes
// S_i(j) also proves PV_i(j-1) finished, which lets softmax group i rescale
// O_i without another barrier.
//
// Softmax works in the log2 domain with lazy rescaling: the running max used
// as exponent base moves only when a row max exceeds it by more than 8
// (2^8 headroom), which is exact because the final 1/l uses the same base.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "sm100.cuh"

namespace gae {

struct AttnParams {
    CUtensorMap tm_q;  // dims {D, Nq, H, B}, box {128 bytes, 128, 1, 1}, 128B swizzle
    CUtensorMap tm_k;  // dims {D, Nkv, H, B}
    CUtensorMap tm_v;
    CUtensorMap tm_ks;      // int8 mode: k_scale as dims {Nkv, B*H}, box {128, 1}
    const float *q_scale;   // int8 mode: [B*H, Nq]
    void *o;
    float *lse;
    int64_t o_sb, o_sh, o_ss;  // element strides of O
    int B, H, Nq, Nkv;
    int n_qpairs;
    int head_major;  // unit order: 1 = all query blocks of a head in a row, 0 = heaviest first
    int causal;
    float scale_log2;  // scale * log2(e)
    int64_t q_offset, kv_offset;
    // int8 mode, diagnostics (the kDump instantiation): every softmax thread
    // also writes the exact int32 logits it read from TMEM, [B*H, Nq, Nkv]
    // (tiles wholly above the causal diagonal are never computed).
    int32_t *logits_dump;
};

// Optional cycle-stamp trace of one CTA (diagnostics; see gae_debug.h).  When
// gae_attn_trace is non-null, CTA (trace_cta, 0) records %clock64 at the
// pipeline events below, indexed by K/V tile (up to kTraceTiles).
constexpr int kTraceTiles = 256;
enum TraceEvent : int {
    kTrSWait0 = 0, kTrSWait1, kTrPDone0, kTrPDone1,  // softmax group g: S ready / P written
    kTrMmaP0, kTrMmaP1, kTrMmaIssued0, kTrMmaIssued1,  // MMA warp: P_g seen / MMAs issued
    // per active unit (index = the CTA's unit count): CTA set up (unit 0
    // only), group 0 saw its first S, group 0 epilogue start / end
    kTrCtaStart, kTrUnitFirstS, kTrEpiStart, kTrEpiEnd,
    kTrNumEvents
};
__device__ unsigned long long *gae_attn_trace = nullptr;
__device__ int gae_attn_trace_cta = 0;
#ifdef GAE_ATTN_TRACE
#define GAE_TRACE(ev, tile)                                                     \
    do {                                                                        \
        if (trace && (tile) < kTraceTiles) trace[(ev) * kTraceTiles + (tile)] = clock64_now(); \
    } while (0)
#else
#define GAE_TRACE(ev, tile) do { } while (0)
#endif

__device__ __forceinline__ unsigned long long clock64_now() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%clock64;" : "=l"(t));
    return t;
}

enum AttnWaitSite : unsigned {
    kSiteQ = 0x101,
    kSiteKvFull = 0x102,
    kSiteKvEmpty = 0x103,
    kSiteS = 0x104,
    kSiteP = 0x105,
    kSiteO = 0x106,
    kSiteDone = 0x107,
};

// kModeSymI8: the symphony layer's integer attention at head_dim 256 --
// Q and K int8 rows of 2*D values (QK^T over 256 dimensions on the int8
// tensor cores, exact int32), V, P and O f16 over D = 128 columns (one half
// of the 256-wide V per launch), no per-row query scale (q_scale NULL).
enum AttnMode : int { kModeBF16 = 0, kModeF16 = 1, kModeInt8 = 2, kModeSymI8 = 3 };

template <int D, int kMode>
struct AttnCfg {
    static constexpr bool kInt8 = kMode == kModeInt8 || kMode == kModeSymI8;
    static constexpr int kBlockM = 128;                      // rows per Q tile
    static constexpr int kBlockN = 128;                      // keys per K/V tile
    static constexpr int kBoxBytes = 128 * 128;              // 128 rows x 128 B
    static constexpr int kQKRowBytes = (kMode == kModeInt8) ? D : 2 * D;  // Q/K row
    static constexpr int kQKBoxes = kQKRowBytes / 128;       // 128-byte swizzle boxes per Q/K row
    static constexpr int kVBoxes = D * 2 / 128;              // V is 16-bit in every mode
    static constexpr int kQTileBytes = kQKBoxes * kBoxBytes;
    static constexpr int kKTileBytes = kQKBoxes * kBoxBytes;
    static constexpr int kVTileBytes = kVBoxes * kBoxBytes;
    static constexpr int kKScaleBytes = kInt8 ? kBlockN * 4 : 0;  // per-key scales after K
    // A slot holds a V tile or a K tile with its scales (1024-byte multiple).
    static constexpr int kSlotBytes = (kKTileBytes + kKScaleBytes > kVTileBytes)
                                          ? (kKTileBytes + kKScaleBytes + 1023) / 1024 * 1024
                                          : kVTileBytes;
    static constexpr int kStages = (D == 128) ? (kMode == kModeInt8 ? 5 : 4) : 8;  // K/V ring slots
    static constexpr int kQBytes = 2 * kQTileBytes;  // one unit's two Q tiles
    // Q buffers: at head_dim 64 (persistent grid, short units) the next unit's
    // Q loads while the current one runs; at 128 shared memory allows one.
    static constexpr int kQStages = (D == 64) ? 2 : 1;
    static constexpr int kRingBytes = kStages * kSlotBytes;
    // Row sums by the tensor core (16-bit modes at head_dim 64, where the
    // softmax instruction stream is the bound and the tensor pipe has room):
    // P.V runs with 16 more B columns of ones read from a constant panel, so
    // O's column D accumulates sum(P) -- rescaled with O, from the same
    // rounded P as the numerator -- instead of the softmax warps adding it up.
    static constexpr bool kMmaRowSum = (D == 64) && !kInt8;
    static constexpr int kOCols = D + (kMmaRowSum ? 16 : 0);
    static constexpr int kOnesBytes = kMmaRowSum ? kBoxBytes : 0;
    static constexpr int kOffOnes = kQStages * kQBytes + kRingBytes;
    static constexpr int kBarOffset = kOffOnes + kOnesBytes;
    // barriers: q_full, kv_full[S], kv_empty[S], s_full[2], p_full[2], o_full[2], done, q_empty,
    // q_full / q_empty of the second Q stage
    // P_i * V issued in two halves (head_dim 128: measured +0.4 to +1.6%;
    // at 64 the f16 symphony layer lost 3%, so it stays whole there).
    static constexpr bool kSplitPV = (D == 128);
    // + p_half[2]: the first 64 keys of P_i written
    static constexpr int kNumBars = 1 + 2 * kStages + 2 + 2 + 2 + 1 + 1 + 2 + 2;
    static constexpr int kSmemBytes = kBarOffset + kNumBars * 8 + 16 + 1024;  // +align slack
    static constexpr uint32_t kTmemCols = 512;
    static constexpr uint32_t kColS0 = 0, kColS1 = 128, kColO0 = 256, kColO1 = 256 + kOCols;
    static_assert(256 + 2 * kOCols <= 512, "TMEM budget");
    static constexpr int kThreads = 384;
    // The producer warps' unit loop needs more than 72 registers (96 with the
    // int8 scale loads); the softmax warps take the rest.
    static constexpr int kRegsSoftmax = kInt8 ? 200 : 208, kRegsProducer = kInt8 ? 96 : 80;
    static_assert(2 * 128 * kRegsSoftmax + 128 * kRegsProducer <= kThreads * 168, "register split");
    static_assert(kInt8 ? (D == 128) : (D == 64 || D == 128), "unsupported head_dim");
    static_assert(kKTileBytes + kKScaleBytes <= kSlotBytes, "K slot too small");
    static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

// Every kPeriod-th pair of probabilities can be computed by the polynomial
// exp2 on the FMA pipe instead of the MUFU (0 = never).  Measured on B200:
// the MUFU gives 4 ex2 per cycle per SM sub-partition and the polynomial 3.6
// (issue-bound), and the two pipes run side by side.  At head_dim 128 the
// tensor work per tile equals the MUFU work and moving pairs over did not
// help; at head_dim 64 the tensor work per exponential is halved and the
// kernel is MUFU-bound.
#ifndef GAE_EMU_PERIOD_D128
#define GAE_EMU_PERIOD_D128 0
#endif
#ifndef GAE_EMU_PERIOD_D64
#define GAE_EMU_PERIOD_D64 3
#endif
// int8 mode (head_dim 128): measured on config 3, every 2nd / 3rd / 4th pair
// on the polynomial gave 947 / 1039 / 1022 TFLOP/s against 1148 without.
#ifndef GAE_EMU_PERIOD_INT8
#define GAE_EMU_PERIOD_INT8 0
#endif
template <int D, int kMode>
__device__ __forceinline__ constexpr bool use_poly_exp(int e) {
    constexpr int kPeriod = (kMode == kModeInt8 || kMode == kModeSymI8) ? GAE_EMU_PERIOD_INT8
                            : (D == 64)          ? GAE_EMU_PERIOD_D64
                                                 : GAE_EMU_PERIOD_D128;
    return kPeriod > 0 && (e % (kPeriod > 0 ? kPeriod : 1)) == kPeriod - 1;
}

// kDump (int8 mode, diagnostics): the same kernel also writes the int32
// logits it reads from TMEM to p.logits_dump; a separate instantiation so
// the production kernel carries none of its registers.
template <int D, int kMode, bool kDump = false>
__global__ void __launch_bounds__(384, 1) attn_fwd_sm100_kernel(const __grid_constant__ AttnParams p) {
    using Cfg = AttnCfg<D, kMode>;
    constexpr bool kBF16 = kMode == kModeBF16 || kMode == kModeInt8;  // P and O bf16 (else f16)
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment for the 128B-swizzle atoms.
    const uint32_t raw_addr = smem_u32(smem_raw);
    const uint32_t base = (raw_addr + 1023u) & ~1023u;
    uint8_t *smem = smem_raw + (base - raw_addr);

    auto sQ = [&](int st) { return base + st * Cfg::kQBytes; };
    const uint32_t sRing = base + Cfg::kQStages * Cfg::kQBytes;
    const uint32_t sBar = base + Cfg::kBarOffset;
    auto bar_q = [&](int st) { return st ? sBar + 8u * (9 + 2 * Cfg::kStages) : sBar; };
    auto bar_kv_full = [&](int s) { return sBar + 8u * (1 + s); };
    auto bar_kv_empty = [&](int s) { return sBar + 8u * (1 + Cfg::kStages + s); };
    auto bar_s = [&](int i) { return sBar + 8u * (1 + 2 * Cfg::kStages + i); };
    auto bar_p = [&](int i) { return sBar + 8u * (3 + 2 * Cfg::kStages + i); };
    auto bar_o = [&](int i) { return sBar + 8u * (5 + 2 * Cfg::kStages + i); };
    const uint32_t bar_done = sBar + 8u * (7 + 2 * Cfg::kStages);
    auto bar_q_empty = [&](int st) { return sBar + 8u * (st ? 10 + 2 * Cfg::kStages : 8 + 2 * Cfg::kStages); };
    auto bar_p_half = [&](int i) { return sBar + 8u * (11 + 2 * Cfg::kStages + i); };
    uint32_t *tmem_base_slot = reinterpret_cast<uint32_t *>(smem + Cfg::kBarOffset + Cfg::kNumBars * 8);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_base_slot + 1);

    volatile int no_abort = 0;  // for drains that must not be cut short
#ifdef GAE_ATTN_TRACE
    unsigned long long *trace =
        (gae_attn_trace && blockIdx.x == gae_attn_trace_cta && blockIdx.y == 0) ? gae_attn_trace : nullptr;
#endif
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    // Persistent schedule: the CTAs share out the list of (query pair,
    // batch*head) units, ordered heaviest first (the last query pairs see the most keys under a causal
    // mask).  TMEM, barriers and the K/V ring live across units; barrier
    // phases follow running counters (tiles, ring items, active units) that
    // every role advances identically.
    const int BH = p.B * p.H;
    const int n_units = p.n_qpairs * BH;
    // skip0: under the causal mask the unit's last K/V tile lies wholly above
    // the diagonal of Q tile 0, so group 0 runs one tile fewer than group 1.
    struct Unit { int q0, b, h, bh, n_kv, skip0; };
    auto unit_at = [&](int u) {
        Unit x;
        // head-major keeps the K/V of a head in L2 while its query blocks run
        // side by side; heaviest first balances a persistent grid.
        const int qpair = p.n_qpairs - 1 - (p.head_major ? u % p.n_qpairs : u / BH);
        x.bh = p.head_major ? u / p.n_qpairs : u % BH;
        x.b = x.bh / p.H;
        x.h = x.bh % p.H;
        x.q0 = qpair * 256;
        int n = (p.Nkv + Cfg::kBlockN - 1) / Cfg::kBlockN;
        if (p.causal) {
            const int64_t last_q = p.q_offset + (int64_t)min(x.q0 + 255, p.Nq - 1);
            const int64_t last_key = last_q - p.kv_offset;
            n = (last_key < 0) ? 0 : (int)min64((int64_t)n, last_key / Cfg::kBlockN + 1);
        }
        x.n_kv = n;
        x.skip0 = 0;
        if (p.causal && n >= 2) {
            const int64_t last_q0 = p.q_offset + (int64_t)min(x.q0 + 127, p.Nq - 1);
            x.skip0 = (p.kv_offset + (int64_t)(n - 1) * Cfg::kBlockN > last_q0) ? 1 : 0;
        }
        return x;
    };
    // Serpentine assignment: in round k this CTA takes list entry
    // k*G + c (k even) or k*G + G-1-c (k odd), so the CTA that takes the
    // heaviest entry of one round takes the lightest of the next.
    const int G = gridDim.x, cta = blockIdx.x;
    auto unit_of = [&](int k) { return k * G + ((k & 1) ? (G - 1 - cta) : cta); };
    // Does this CTA have any unit with keys to visit (then it needs TMEM)?
    bool any_work = false;
    for (int k = 0; k * G < n_units && !any_work; ++k)
        if (unit_of(k) < n_units) any_work = unit_at(unit_of(k)).n_kv > 0;

    if (threadIdx.x == 0) {
        for (int st = 0; st < 2; ++st) {
            mbar_init(bar_q(st), 1);
            mbar_init(bar_q_empty(st), 1);
        }
        for (int s = 0; s < Cfg::kStages; ++s) {
            mbar_init(bar_kv_full(s), 1);
            mbar_init(bar_kv_empty(s), 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(bar_s(i), 1);
            mbar_init(bar_p(i), 128);
            mbar_init(bar_p_half(i), 128);
            mbar_init(bar_o(i), 1);
        }
        mbar_init(bar_done, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if constexpr (Cfg::kMmaRowSum) {
        // The constant B panel of ones (whole panel, so the swizzle is moot).
        const uint32_t one2 = kBF16 ? 0x3F803F80u : 0x3C003C00u;
        uint4 *ones = reinterpret_cast<uint4 *>(smem + Cfg::kOffOnes);
        for (int i = threadIdx.x; i < Cfg::kOnesBytes / 16; i += blockDim.x)
            ones[i] = make_uint4(one2, one2, one2, one2);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 9 && any_work) {
        tmem_alloc(smem_u32(tmem_base_slot), Cfg::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = any_work ? *tmem_base_slot : 0u;
    if (threadIdx.x == 0) GAE_TRACE(kTrCtaStart, 0);

    if (warp >= 10) {
        regs_dec<Cfg::kRegsProducer>();
    } else if (warp == 8) {
        // ------------------------------------------------------ TMA producer
        regs_dec<Cfg::kRegsProducer>();
        if (lane == 0 && any_work) {
            tma_prefetch_desc(&p.tm_q);
            tma_prefetch_desc(&p.tm_k);
            tma_prefetch_desc(&p.tm_v);
            if (Cfg::kInt8) tma_prefetch_desc(&p.tm_ks);
            bool ok = true;
            int item = 0;  // running ring item (K_j, V_j, K_j+1, ...)
            int au = 0;    // running active unit
            auto load_item = [&](const Unit &x, int j, int kv) {
                const int slot = item % Cfg::kStages, use = item / Cfg::kStages;
                if (use > 0 && !(ok = mbar_wait(bar_kv_empty(slot), (use - 1) & 1, kSiteKvEmpty, abort_flag)))
                    return;
                const uint32_t dst = sRing + slot * Cfg::kSlotBytes;
                if (kv) {
                    mbar_expect_tx(bar_kv_full(slot), Cfg::kVTileBytes);
                    for (int hf = 0; hf < Cfg::kVBoxes; ++hf)
                        tma_load_4d(dst + hf * Cfg::kBoxBytes, &p.tm_v, bar_kv_full(slot), hf * 64,
                                    j * Cfg::kBlockN, x.h, x.b);
                } else {
                    mbar_expect_tx(bar_kv_full(slot), Cfg::kKTileBytes + Cfg::kKScaleBytes);
                    for (int hf = 0; hf < Cfg::kQKBoxes; ++hf)
                        tma_load_4d(dst + hf * Cfg::kBoxBytes, &p.tm_k, bar_kv_full(slot),
                                    hf * 128 / (Cfg::kInt8 ? 1 : 2), j * Cfg::kBlockN, x.h, x.b);
                    if (Cfg::kInt8)
                        tma_load_2d(dst + Cfg::kKTileBytes, &p.tm_ks, bar_kv_full(slot), j * Cfg::kBlockN, x.bh);
                }
                ++item;
            };
            for (int k = 0; k * G < n_units && ok; ++k) {
                const int u = unit_of(k);
                if (u >= n_units) continue;
                const Unit x = unit_at(u);
                if (x.n_kv == 0) continue;
                // K_0, V_0 first: they only need free ring slots, while Q waits
                // for the last QK^T of the unit that used its stage before.
                for (int it = 0; it < 2 && ok; ++it) load_item(x, 0, it);
                if (!ok) break;
                const int qs = au % Cfg::kQStages, qu = au / Cfg::kQStages;  // stage, its use
                if (qu > 0 && !(ok = mbar_wait(bar_q_empty(qs), (qu - 1) & 1, kSiteQ, abort_flag))) break;
                mbar_expect_tx(bar_q(qs), Cfg::kQBytes);
                for (int t = 0; t < 2; ++t)
                    for (int hf = 0; hf < Cfg::kQKBoxes; ++hf)
                        tma_load_4d(sQ(qs) + t * Cfg::kQTileBytes + hf * Cfg::kBoxBytes, &p.tm_q, bar_q(qs),
                                    hf * 128 / (Cfg::kInt8 ? 1 : 2), x.q0 + t * 128, x.h, x.b);
                for (int j = 1; j < x.n_kv && ok; ++j)
                    for (int kv = 0; kv < 2 && ok; ++kv) load_item(x, j, kv);
                ++au;
            }
            // Drain: the last Q and the last copy issued into each slot have
            // landed before the CTA can exit (bounded; normally complete).
            for (int a = max(0, au - Cfg::kQStages); a < au; ++a)
                mbar_wait(bar_q(a % Cfg::kQStages), (a / Cfg::kQStages) & 1, kSiteQ, &no_abort);
            for (int i = max(0, item - Cfg::kStages); i < item; ++i)
                mbar_wait(bar_kv_full(i % Cfg::kStages), (i / Cfg::kStages) & 1, kSiteKvFull, &no_abort);
        }
    } else if (warp == 9) {
        // ---------------------------------------------------------- MMA issuer
        regs_dec<Cfg::kRegsProducer>();
        if (lane == 0 && any_work) {
            constexpr uint32_t idesc_qk =
                Cfg::kInt8 ? idesc_i8(128, 128) : idesc_f16(128, 128, kBF16, false, false);
            constexpr uint32_t idesc_pv = idesc_f16(128, Cfg::kOCols, kBF16, false, true);
            auto issue_qk = [&](int i, int slot, uint32_t q_base) {
                const uint32_t d_tmem = tmem + (i ? Cfg::kColS1 : Cfg::kColS0);
                const uint32_t qa = q_base + i * Cfg::kQTileBytes;
                const uint32_t kb = sRing + slot * Cfg::kSlotBytes;
                // One MMA consumes 32 bytes of K (16 bf16 or 32 int8 elements).
#pragma unroll
                for (int kk = 0; kk < Cfg::kQKRowBytes / 32; ++kk) {
                    const uint32_t off = (kk >> 2) * Cfg::kBoxBytes + (kk & 3) * 32;
                    if constexpr (Cfg::kInt8)
                        umma_i8_ss(d_tmem, smem_desc_sw128(qa + off, 16, 1024),
                                   smem_desc_sw128(kb + off, 16, 1024), idesc_qk, kk > 0);
                    else
                        umma_f16_ss(d_tmem, smem_desc_sw128(qa + off, 16, 1024),
                                    smem_desc_sw128(kb + off, 16, 1024), idesc_qk, kk > 0);
                }
            };
            // P_i * V in two halves of 64 keys: the first is issued as soon
            // as the softmax group has written the first half of P_i (while
            // it still computes the second), the second once all of P_i is
            // there.  ph: phase parity of this tile's p_half / p_full.
            auto issue_pv = [&](int i, int slot, bool acc, int ph, int tr) -> bool {
                const uint32_t d_tmem = tmem + (i ? Cfg::kColO1 : Cfg::kColO0);
                const uint32_t p_tmem = tmem + (i ? Cfg::kColS1 : Cfg::kColS0);
                const uint32_t vb = sRing + slot * Cfg::kSlotBytes;
                (void)tr;
                if constexpr (!Cfg::kSplitPV) {
                    if (!mbar_wait(bar_p(i), ph, kSiteP, abort_flag)) return false;
                    if (tr >= 0) GAE_TRACE(kTrMmaP0 + i, tr);
                    tc_fence_after();
#pragma unroll
                    for (int kk = 0; kk < Cfg::kBlockN / 16; ++kk)
                        umma_f16_ts(d_tmem, p_tmem + kk * 8,
                                    smem_desc_sw128(vb + kk * 16 * 128,
                                                    Cfg::kMmaRowSum ? (base + Cfg::kOffOnes) - vb : Cfg::kBoxBytes,
                                                    1024),
                                    idesc_pv, (acc || kk > 0) ? 1u : 0u);
                    return true;
                }
                constexpr int kHalves = Cfg::kSplitPV ? 2 : 1;
                for (int h = 0; h < kHalves; ++h) {
                    if (!mbar_wait((h || !Cfg::kSplitPV) ? bar_p(i) : bar_p_half(i), ph, kSiteP, abort_flag))
                        return false;
                    if (h == 0 && tr >= 0) GAE_TRACE(kTrMmaP0 + i, tr);
                    tc_fence_after();
#pragma unroll
                    for (int k2 = 0; k2 < Cfg::kBlockN / 16 / kHalves; ++k2) {
                        const int kk = h * (Cfg::kBlockN / 16 / kHalves) + k2;
                        umma_f16_ts(d_tmem, p_tmem + kk * 8,
                                    smem_desc_sw128(vb + kk * 16 * 128,
                                                    Cfg::kMmaRowSum ? (base + Cfg::kOffOnes) - vb : Cfg::kBoxBytes,
                                                    1024),
                                    idesc_pv, (acc || kk > 0) ? 1u : 0u);
                    }
                }
                return true;
            };
            bool ok = true;
            int ib = 0;  // ring item of this unit's K_0
            int gt0 = 0, gt1 = 0;  // running tiles of groups 0 / 1 (phase of s_full / p_full)
            bool early_qk0 = false;  // this unit's QK0 of tile 0 was issued during the previous unit
            int au = 0;            // running active unit (phase of q_full / q_empty / o_full)
            for (int k = 0; k * G < n_units && ok; ++k) {
                const int u = unit_of(k);
                if (u >= n_units) continue;
                const Unit x = unit_at(u);
                const int n_kv = x.n_kv;
                if (n_kv == 0) continue;
                const int qs = au % Cfg::kQStages;
                const uint32_t q_base = sQ(qs);
                if (!(ok = mbar_wait(bar_q(qs), (au / Cfg::kQStages) & 1, kSiteQ, abort_flag))) break;
                for (int j = 0; j < n_kv && ok; ++j) {
                    const int k_item = ib + 2 * j, k_slot = k_item % Cfg::kStages;
                    const int v_item = ib + 2 * j - 1, v_slot = v_item % Cfg::kStages;
                    ok = mbar_wait(bar_kv_full(k_slot), (k_item / Cfg::kStages) & 1, kSiteKvFull, abort_flag);
                    if (!ok) break;
                    if (j > 0) {
                        ok = mbar_wait(bar_kv_full(v_slot), (v_item / Cfg::kStages) & 1, kSiteKvFull, abort_flag) &&
                             issue_pv(0, v_slot, j - 1 > 0, (gt0 + j - 1) & 1, au == 0 ? j - 1 : -1);
                        if (!ok) break;
                    }
                    if (!(x.skip0 && j == n_kv - 1) && !(early_qk0 && j == 0)) {
                        issue_qk(0, k_slot, q_base);
                        umma_commit(bar_s(0));
                    }
                    if (au == 0) GAE_TRACE(kTrMmaIssued0, j);
                    if (j > 0) {
                        ok = issue_pv(1, v_slot, j - 1 > 0, (gt1 + j - 1) & 1, au == 0 ? j - 1 : -1);
                        if (!ok) break;
                        umma_commit(bar_kv_empty(v_slot));
                        // int8: both softmax groups have read K_{j-1}'s scales from its slot.
                        if (Cfg::kInt8) mbar_arrive(bar_kv_empty((k_item - 2) % Cfg::kStages));
                    }
                    issue_qk(1, k_slot, q_base);
                    umma_commit(bar_s(1));
                    if (!Cfg::kInt8) umma_commit(bar_kv_empty(k_slot));
                    if (j == n_kv - 1) umma_commit(bar_q_empty(qs));  // Q may be reloaded after this
                    if (au == 0) GAE_TRACE(kTrMmaIssued1, j);
                }
                if (!ok) break;
                const int v_item = ib + 2 * n_kv - 1, v_slot = v_item % Cfg::kStages;
                if (!(ok = mbar_wait(bar_kv_full(v_slot), (v_item / Cfg::kStages) & 1, kSiteKvFull, abort_flag)))
                    break;
                if (x.skip0) {
                    umma_commit(bar_o(0));  // PV0 of its last tile was issued in the loop
                } else {
                    if (!(ok = issue_pv(0, v_slot, n_kv > 1, (gt0 + n_kv - 1) & 1, -1))) break;
                    umma_commit(bar_o(0));
                }
                // Group 0 is done with this unit while group 1 still works on its
                // last tile: if the next unit's Q and K_0 have landed, start its
                // first QK0 now (S0 was released with group 0's last P; tcgen05
                // MMAs of this thread run in issue order, so the PV0 above reads
                // it first).  Only probes, so group 1's last tile never waits.
                early_qk0 = false;
                for (int k2 = k + 1; k2 * G < n_units; ++k2) {
                    const int u2 = unit_of(k2);
                    if (u2 >= n_units || unit_at(u2).n_kv == 0) continue;
                    const int qs2 = (au + 1) % Cfg::kQStages;
                    const int k2_item = ib + 2 * n_kv, k2_slot = k2_item % Cfg::kStages;
                    if (mbar_test(bar_q(qs2), ((au + 1) / Cfg::kQStages) & 1) &&
                        mbar_test(bar_kv_full(k2_slot), (k2_item / Cfg::kStages) & 1)) {
                        tc_fence_after();
                        issue_qk(0, k2_slot, sQ(qs2));
                        umma_commit(bar_s(0));
                        early_qk0 = true;
                    }
                    break;
                }
                if (!(ok = issue_pv(1, v_slot, n_kv > 1, (gt1 + n_kv - 1) & 1, -1))) break;
                umma_commit(bar_o(1));
                umma_commit(bar_kv_empty(v_slot));
                if (Cfg::kInt8) mbar_arrive(bar_kv_empty((v_item - 1) % Cfg::kStages));
                ib += 2 * n_kv;
                gt0 += n_kv - x.skip0;
                gt1 += n_kv;
                ++au;
            }
            // Drain: every MMA this thread issued has completed before TMEM is
            // freed (bounded, and not cut short by the abort flag).
            umma_commit(bar_done);
            mbar_wait(bar_done, 0, kSiteDone, &no_abort);
        }
    } else {
        // ------------------------------------------------------ softmax groups
        regs_inc<Cfg::kRegsSoftmax>();
        const int grp = warp >> 2;       // Q tile 0 or 1
        const int wq = warp & 3;         // TMEM lane quarter
        const int row = wq * 32 + lane;  // row within the Q tile
        const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
        const uint32_t tS = tmem + lane_off + (grp ? Cfg::kColS1 : Cfg::kColS0);
        const uint32_t tO = tmem + lane_off + (grp ? Cfg::kColO1 : Cfg::kColO0);
        bool ok = true;
        int ib = 0, gt = 0, au = 0;  // same running counters as the MMA issuer
        for (int k = 0; k * G < n_units && ok; ++k) {
                const int u = unit_of(k);
                if (u >= n_units) continue;
        const Unit x = unit_at(u);
        const int n_kv = x.n_kv, b = x.b, h = x.h, bh = x.bh;
        const int n_mine = n_kv - (grp == 0 ? x.skip0 : 0);  // K/V tiles this group processes
        const int q_local = x.q0 + grp * 128 + row;
        const int64_t q_abs = p.q_offset + q_local;
        // Factor that takes a raw score to the log2 domain: scale*log2(e), times
        // the query row's dequantisation scale in int8 mode.
        float sl2 = p.scale_log2;
        if constexpr (Cfg::kInt8)
            sl2 *= (q_local < p.Nq) ? (p.q_scale ? p.q_scale[(int64_t)bh * p.Nq + q_local] : 1.f) : 0.f;
        // A zero factor (zero scale, or an all-zero int8 query row) makes every
        // visible score equal; a tiny positive factor keeps that result while
        // masked (-inf) entries still map to probability 0 instead of NaN.
        sl2 = fmaxf(sl2, 1e-30f);

        float m_run = -INFINITY;  // exponent base, log2 domain (scaled)
        float l_run = 0.f;
        for (int j = 0; j < n_mine; ++j) {
            ok = mbar_wait(bar_s(grp), (gt + j) & 1, kSiteS, abort_flag);
            if (!ok) break;
            if (row == 0 && au == 0) GAE_TRACE(kTrSWait0 + grp, j);
            if (row == 0 && grp == 0 && j == 0) GAE_TRACE(kTrUnitFirstS, au);
            tc_fence_after();
            float s[128];
            {
                uint32_t r0[32], r1[32], r2[32], r3[32];
                tmem_ld32(tS + 0, r0);
                tmem_ld32(tS + 32, r1);
                tmem_ld32(tS + 64, r2);
                tmem_ld32(tS + 96, r3);
                tmem_wait_ld();
                if constexpr (Cfg::kInt8) {
                    if (kDump && q_local < p.Nq) {
                        int32_t *dst = p.logits_dump + ((int64_t)bh * p.Nq + q_local) * p.Nkv +
                                       (int64_t)j * Cfg::kBlockN;
                        const int nk = min(Cfg::kBlockN, p.Nkv - j * Cfg::kBlockN);
#pragma unroll
                        for (int e = 0; e < 32; ++e) {  // constant register indices
                            if (e < nk) dst[e] = (int32_t)r0[e];
                            if (32 + e < nk) dst[32 + e] = (int32_t)r1[e];
                            if (64 + e < nk) dst[64 + e] = (int32_t)r2[e];
                            if (96 + e < nk) dst[96 + e] = (int32_t)r3[e];
                        }
                    }
                    // Exact int32 logits times the keys' dequantisation scales.  The
                    // scales arrived with K_j; its slot is released only after both
                    // softmax groups finished tile j.
                    const int slot = (ib + 2 * j) % Cfg::kStages;
                    if (!mbar_wait(bar_kv_full(slot), ((ib + 2 * j) / Cfg::kStages) & 1, kSiteKvFull,
                                   abort_flag)) {
                        ok = false;
                        break;
                    }
                    const float4 *ks = reinterpret_cast<const float4 *>(
                        smem + Cfg::kQStages * Cfg::kQBytes + slot * Cfg::kSlotBytes + Cfg::kKTileBytes);
#pragma unroll
                    for (int e4 = 0; e4 < 8; ++e4) {
                        const float4 a = ks[e4], bq = ks[8 + e4], c = ks[16 + e4], d = ks[24 + e4];
                        const float ka[4] = {a.x, a.y, a.z, a.w}, kb4[4] = {bq.x, bq.y, bq.z, bq.w};
                        const float kc[4] = {c.x, c.y, c.z, c.w}, kd[4] = {d.x, d.y, d.z, d.w};
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            s[4 * e4 + u] = (float)(int)r0[4 * e4 + u] * ka[u];
                            s[32 + 4 * e4 + u] = (float)(int)r1[4 * e4 + u] * kb4[u];
                            s[64 + 4 * e4 + u] = (float)(int)r2[4 * e4 + u] * kc[u];
                            s[96 + 4 * e4 + u] = (float)(int)r3[4 * e4 + u] * kd[u];
                        }
                    }
                } else {
#pragma unroll
                    for (int e = 0; e < 32; ++e) {
                        s[e] = __uint_as_float(r0[e]);
                        s[32 + e] = __uint_as_float(r1[e]);
                        s[64 + e] = __uint_as_float(r2[e]);
                        s[96 + e] = __uint_as_float(r3[e]);
                    }
                }
            }
            // Masking: causal boundary and the ragged end of the key range.
            const int64_t k_abs0 = p.kv_offset + (int64_t)j * Cfg::kBlockN;
            int limit = min(Cfg::kBlockN, p.Nkv - j * Cfg::kBlockN);
            if (p.causal) {
                const int64_t lim_c = q_abs - k_abs0 + 1;
                if (lim_c < limit) limit = (int)max64(lim_c, 0);
            }
            if (limit < Cfg::kBlockN) {
#pragma unroll
                for (int c = 0; c < 128; ++c) s[c] = (c < limit) ? s[c] : -INFINITY;
            }
            // Row max: four independent chains of three-input max.
            float mq[4];
#pragma unroll
            for (int k4 = 0; k4 < 4; ++k4) {
                float m = s[32 * k4];
#pragma unroll
                for (int i = 1; i < 31; i += 2) m = fmax3(m, s[32 * k4 + i], s[32 * k4 + i + 1]);
                mq[k4] = fmaxf(m, s[32 * k4 + 31]);
            }
            const float mx = fmax3(fmaxf(mq[0], mq[1]), mq[2], mq[3]);
            const float m_tile = (mx == -INFINITY) ? -INFINITY : mx * sl2;
            float alpha = 1.f;
            if (m_tile > m_run + 8.f) {  // also true while m_run == -inf and the tile sees a key
                alpha = (m_run == -INFINITY) ? 0.f : ex2_approx(m_run - m_tile);
                m_run = m_tile;
            }
            // Does O_i need rescaling this tile (warp-uniform)?  Then the
            // first half of P_i is published only after the rescale below.
            const bool rescale = Cfg::kSplitPV && j > 0 && __any_sync(0xffffffffu, alpha != 1.f);
            const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
            // p = 2^(s*sl2 - m): packed fp32x2 FMA, MUFU ex2, packed partial sums
            // (four independent pair accumulators).
            const uint64_t sl2x2 = f2_pack(sl2, sl2), negm2 = f2_pack(-m_use, -m_use);
            uint64_t acc2[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                uint32_t pk[16];
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    const uint64_t x = f2_fma(f2_pack(s[c * 32 + 2 * e], s[c * 32 + 2 * e + 1]), sl2x2, negm2);
                    float p0, p1;
                    if (use_poly_exp<D, kMode>(e)) {
                        exp2_poly_x2(x, p0, p1);  // this pair on the FMA pipe
                    } else {
                        float x0, x1;
                        f2_unpack(x, x0, x1);
                        p0 = ex2_approx(x0);
                        p1 = ex2_approx(x1);
                    }
                    acc2[e & 3] = f2_add(acc2[e & 3], f2_pack(p0, p1));
                    pk[e] = kBF16 ? pack_bf16x2(p0, p1) : pack_f16x2(p0, p1);
                }
                tmem_st16(tS + c * 16, pk);
                if (Cfg::kSplitPV && c == 1 && !rescale) {  // the first 64 keys of P_i: their half of P_i * V may start
                    tmem_wait_st();
                    tc_fence_before();
                    mbar_arrive(bar_p_half(grp));
                }
            }
            if constexpr (!Cfg::kMmaRowSum) {
                float a0, a1;
                f2_unpack(f2_add(f2_add(acc2[0], acc2[1]), f2_add(acc2[2], acc2[3])), a0, a1);
                l_run = l_run * alpha + (a0 + a1);
            } else {
                (void)acc2;
            }
            // Rescale O_i when the base moved (warp-uniform: tcgen05.ld/st are
            // warp-collective), before any of this tile's P*V is issued.
            // PV_i(j-1) has completed: its commit preceded S_i(j)'s.
            if (Cfg::kSplitPV ? rescale : (j > 0 && __any_sync(0xffffffffu, alpha != 1.f))) {
#pragma unroll
                for (int c = 0; c < D / 32; ++c) {
                    uint32_t r[32];
                    tmem_ld32(tO + c * 32, r);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * alpha);
                    tmem_st32(tO + c * 32, r);
                }
                if constexpr (Cfg::kMmaRowSum) {  // the row-sum columns
                    uint32_t r[16];
                    tmem_ld16(tO + D, r);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 16; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * alpha);
                    tmem_st16(tO + D, r);
                }
            }
            tmem_wait_st();
            tc_fence_before();
            if (Cfg::kSplitPV && rescale) mbar_arrive(bar_p_half(grp));
            mbar_arrive(bar_p(grp));
            if (row == 0 && au == 0) GAE_TRACE(kTrPDone0 + grp, j);
        }
        if (!ok) break;

        // Epilogue: O_i / l -> global; log-sum-exp.
        const bool row_valid = q_local < p.Nq;
        if (row == 0 && grp == 0) GAE_TRACE(kTrEpiStart, au);
        if (n_kv > 0 && ok) ok = mbar_wait(bar_o(grp), au & 1, kSiteO, abort_flag);
        if constexpr (Cfg::kMmaRowSum) {
            l_run = 0.f;
            if (n_kv > 0 && ok) {
                tc_fence_after();
                uint32_t r[16];
                tmem_ld16(tO + D, r);
                tmem_wait_ld();
                l_run = __uint_as_float(r[0]);
            }
        }
        const float inv_l = (l_run > 0.f) ? 1.f / l_run : 0.f;
        if (n_kv > 0 && ok) {
            tc_fence_after();
            char *orow = reinterpret_cast<char *>(p.o) +
                         2 * (b * p.o_sb + h * p.o_sh + (int64_t)q_local * p.o_ss);
#pragma unroll
            for (int c = 0; c < D / 32; ++c) {
                uint32_t r[32];
                tmem_ld32(tO + c * 32, r);
                tmem_wait_ld();
                uint32_t pk[16];
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    const float a0 = __uint_as_float(r[2 * e]) * inv_l;
                    const float a1 = __uint_as_float(r[2 * e + 1]) * inv_l;
                    pk[e] = kBF16 ? pack_bf16x2(a0, a1) : pack_f16x2(a0, a1);
                }
                if (row_valid) {
                    uint4 *dst = reinterpret_cast<uint4 *>(orow + c * 64);
#pragma unroll
                    for (int v = 0; v < 4; ++v)
                        dst[v] = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
                }
            }
        } else if (n_kv == 0 && row_valid) {
            char *orow = reinterpret_cast<char *>(p.o) +
                         2 * (b * p.o_sb + h * p.o_sh + (int64_t)q_local * p.o_ss);
            for (int c = 0; c < D / 8; ++c) reinterpret_cast<uint4 *>(orow)[c] = make_uint4(0, 0, 0, 0);
        }
        if (row == 0 && grp == 0) GAE_TRACE(kTrEpiEnd, au);
        if (p.lse && row_valid) {
            float lse = -INFINITY;
            if (l_run > 0.f) lse = (m_run + __log2f(l_run)) * 0.69314718055994531f;
            p.lse[(int64_t)bh * p.Nq + q_local] = lse;
        }
        if (n_kv > 0) {
            ib += 2 * n_kv;
            gt += n_mine;
            ++au;
        }
        }  // units
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 9 && any_work) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, Cfg::kTmemCols);
    }
}

}  // namespace gae
