// FlashAttention-2 forward for Blackwell (sm_100a): TMA + tcgen05 + TMEM, warp specialised.
//
// Reference path being replaced (roy6n23/triton-fa2-forward):
//   fa2/kernel.py:110-183  _attn_fwd        (program = one Q tile of one (batch, q-head))
//   fa2/kernel.py:60-107   _attn_fwd_inner  (per K/V tile: S = QK^T, mask, online softmax, PV)
//   fa2/kernel.py:210-260  attention()      (validation, pack decision, launch)
//
// A work unit is two Q tiles of 128 rows (256 rows; with GQA packing a row is a
// (position, head) pair, row r -> position r / PACK, head r % PACK, fa2/kernel.py:135-141)
// of one (batch, q-head block); it walks the K/V tiles [0, J) it can see, in increasing
// order (the reference's order: stage 1 unmasked tiles from column 0, then the diagonal
// band, nothing to its right; fa2/kernel.py:150-175).
// The launch is persistent: one CTA per SM walks a static list of units (heaviest causal
// row blocks first, snake order over the CTAs). The K/V ring, the TMEM accumulators and the
// barrier phases carry over from one unit to the next, so the next unit's Q and K_0 load
// and its first QK GEMMs run while the softmax warps finish and store the previous unit.
// (With split-KV the grid has one CTA per (unit, split) instead.)
//
// Warp roles (384 threads, three warpgroups):
//   warps 0-3   softmax for Q tile 0   (thread = one row = one TMEM lane; warp w reaches
//               lane quadrant w % 4, the lanes of its SMSP)
//   warps 4-7   softmax for Q tile 1
//   warp  8     tcgen05 MMA issue (one thread) + TMEM allocation
//   warp  9     TMA producer (one thread)
//   warps 10-11 idle (with FA2_TWO_ISSUERS=1, warp 10 issues Q tile 1's MMAs)
// Registers: launched at 168/thread; setmaxnreg moves them to the softmax warpgroups
// (200 each) from the MMA/TMA warpgroup (104): 2 * 200 + 104 == 3 * 168.
// (FA2_ROW_SPLIT=2, a measured-slower alternative: 640 threads, two softmax warps per lane
// quadrant with 64 scores each, warps 16-19 MMA / TMA / spare.)
// TMEM (512 columns x 128 lanes, fp32):  S0 [0,128) S1 [128,256) O0 [256,256+D) O1 [..+D)
//   P_t (fp16/bf16, packed 2 per column) overwrites the upper half of S_t, and the second
//   GEMM reads it straight from TMEM (tcgen05.mma A-from-TMEM).
// MMA order per K/V step j:  PV(0,j) QK(0,j+1) PV(1,j) QK(1,j+1)  -- while softmax 0 works
//   on S0 the tensor core runs tile 1's GEMMs and vice versa (ping-pong).
//
// Online softmax (fa2/kernel.py:90-106) in base 2 with one FFMA per score,
// p = exp2(s * qk_scale - m); l and O accumulate in fp32; P is rounded to the input dtype
// before the PV GEMM (fa2/kernel.py:104-105). The running max is only moved when a row's
// max grows by more than 2^8 (the O and l rescale is then skipped exactly, alpha == 1); the
// final O / l is unchanged because O and l always share the same reference max.
//
// Every mbarrier wait is bounded (mbar_wait); a role that gives up raises FA2_ERR_TIMEOUT
// in the caller's error word and joins the common teardown, so no wait can hang the GPU.

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdint>
#include <cstring>

#include "exp2_poly.cuh"
#include "fa2_sm100.h"
#include "ptx_sm100.cuh"

namespace fa2 {

constexpr int BM = 128;  // rows per Q tile (one TMEM lane each)
constexpr int BN = 128;  // K/V rows per tile
constexpr int Q_TILES = 2;
#ifndef FA2_ROW_SPLIT
// Softmax warps per TMEM lane quadrant of a Q tile. 1: one warp takes all 128 scores of its
// 32 rows (12 warps: 8 softmax, MMA, TMA, 2 spare). 2: two warps take 64 scores each and
// exchange the row max and row sum through TMEM (20 warps: 16 softmax, MMA, TMA, 2 spare).
#define FA2_ROW_SPLIT 1
#endif
#ifndef FA2_RS2_REGS_SOFTMAX
#define FA2_RS2_REGS_SOFTMAX 104  // with FA2_ROW_SPLIT=2; the other warpgroup gets what is left (64)
#endif
constexpr int HALVES = FA2_ROW_SPLIT;
static_assert(HALVES == 1 || HALVES == 2, "row split");
constexpr int SCOLS = BN / HALVES;  // scores of a row per softmax warp
constexpr int SOFTMAX_WARPS = 8 * HALVES;
constexpr int MMA_WARP = SOFTMAX_WARPS;
constexpr int LOAD_WARP = SOFTMAX_WARPS + 1;
constexpr int MMA_WARP2 = SOFTMAX_WARPS + 2;  // second MMA issuer (Q tile 1) with FA2_TWO_ISSUERS
constexpr int NUM_WARPS = HALVES == 1 ? 12 : 20;  // whole warpgroups (setmaxnreg works on warpgroups)
constexpr int NUM_THREADS = NUM_WARPS * 32;
constexpr int TMEM_COLS = 512;
// Softmax warps' registers in the 12-warp layout, per head dim (the MMA/TMA warpgroup gets
// 504 - 2x). Measured: 208 at D = 128 leaves the MMA thread spilling, -6.5%.
#ifndef FA2_REGS_SOFTMAX_D128
#define FA2_REGS_SOFTMAX_D128 200
#endif
#ifndef FA2_REGS_SOFTMAX_D64
#define FA2_REGS_SOFTMAX_D64 192
#endif
// Columns per tcgen05.ld when a softmax warp loads its scores (32, 64 or 128), per head dim.
// Measured: one 128-column load at D = 64 fp16 gave +2.8%, +3.6% and -0.3% on three boxes (bf16
// unchanged); at D = 128 it is -0.2%, and 64-column loads are -4%.
#ifndef FA2_S_LOAD_X_D128
#define FA2_S_LOAD_X_D128 32
#endif
#ifndef FA2_S_LOAD_X_D64
#define FA2_S_LOAD_X_D64 128
#endif
// Launched at REGS_LAUNCH registers a thread (the launch bound's share: 65536 / 384 -> 168,
// and with 20 warps five per SMSP, 16384 / 160 -> 96); setmaxnreg then moves registers from
// the MMA/TMA warpgroup to the softmax warpgroups. The new counts must fit in what the CTA
// was launched with (regs_fit below).
constexpr int REGS_LAUNCH = HALVES == 1 ? 168 : 96;
template <int D>
__host__ __device__ constexpr int regs_softmax() {
  return HALVES == 2 ? FA2_RS2_REGS_SOFTMAX : (D == 128 ? FA2_REGS_SOFTMAX_D128 : FA2_REGS_SOFTMAX_D64);
}
template <int D>
__host__ __device__ constexpr int regs_other() {
  return ((NUM_WARPS * REGS_LAUNCH - SOFTMAX_WARPS * regs_softmax<D>()) / (NUM_WARPS - SOFTMAX_WARPS)) & ~7;
}
template <int D>
__host__ __device__ constexpr int s_load_x() {
  return D == 128 ? FA2_S_LOAD_X_D128 : FA2_S_LOAD_X_D64;
}
#ifndef FA2_RESCALE_TH
#define FA2_RESCALE_TH 8.0f
#endif
constexpr float RESCALE_TH = FA2_RESCALE_TH;     // log2 units: P may reach 2^8 before a rescale
constexpr long long DEFAULT_TIMEOUT = 2000000000LL;  // SM clocks, ~1 s
// Which of the 16 exp2 pairs of a 32-column chunk run on the FMA pipe (the rest on the MUFU).
// D = 128: pairs 7 and 15, i.e. 12.5% on the FMA pipe. With the warp-voted softmax waits this
// measured +0.5..0.6% (headline), +0.8% (mha_causal), +1.4..1.8% (pack_tail) over pairs 3, 7, 11,
// 15 (25%, shipped before; the share FA4 also uses is 12.5%); 3 pairs (18.75%) were in between
// and 37.5% is 6% slower. D = 64 has half the tensor work per score and less pipe headroom for the
// polynomial: pairs 7 and 15 (12.5%) on the FMA pipe, for bf16 (degree-3 polynomial, +7% over
// all-MUFU) and fp16 (+5%); 25% is slower for both.
#ifndef FA2_POLY_DEG_FP16
// Degree of the FMA-pipe exp2 polynomial when P is rounded to fp16. Degree 3 (max rel. error
// 7.5e-5, below half an fp16 ulp, 2^-11 = 4.9e-4) measured +2.6% at D = 64 over degree 4 (2.7e-6).
#define FA2_POLY_DEG_FP16 3
#endif
#ifndef FA2_EMU_MASK_D128
#define FA2_EMU_MASK_D128 0x8080u
#endif
#ifndef FA2_EMU_MASK_D64
#define FA2_EMU_MASK_D64 0x8080u
#endif
#ifndef FA2_EMU_MASK_D64_BF16
#define FA2_EMU_MASK_D64_BF16 0x8080u
#endif
#ifndef FA2_P_SPLIT
#define FA2_P_SPLIT 3  // P chunks (of 32 columns) handed to the MMA warp before the rest
#endif
#ifndef FA2_MMA_SPIN
#define FA2_MMA_SPIN 0  // 1: the MMA thread polls its barriers without suspending (measured: no gain)
#endif
// Speculative max, per head dim. 1: on unmasked steps with a finite reference max, P is
// computed with the current reference max while the row max is taken; a row whose max moves
// past the threshold (rare after the first tile) redoes its P before the hand-off. Same values
// as taking the max first. Measured +4..6% at D = 64 (non-causal); at D = 128 it is within
// +-1% and its redo path keeps the scores live next to the P chunks, which spills registers
// (80-92 bytes on every bf16 build), so D = 128 takes the max first.
#ifndef FA2_SPEC_MAX_D128
#define FA2_SPEC_MAX_D128 0
#endif
#ifndef FA2_SPEC_MAX_D64
#define FA2_SPEC_MAX_D64 1
#endif
#ifndef FA2_STAGES_D128
// K/V ring slots of 32 KiB at D = 128 (the split-KV build uses 4). A 4th slot fits only with
// one O staging chunk per warp (FA2_STG_FULL 0): measured 1-2% slower on the headline with an
// earlier build; with the current kernel, two boxes, two runs each: headline -0.2..+0.2%,
// pack_tail +0.7..1.9%, mha_causal 0..+0.4%, MQA 0, non-causal D = 128 -0.5..-0.7%. 2 is 3% slower.
#define FA2_STAGES_D128 3
#endif
#ifndef FA2_STAGES_D64
#define FA2_STAGES_D64 8   // K/V ring slots of 16 KiB at D = 64
#endif
#ifndef FA2_STG_FULL
// 1: each softmax warp stages all of its 32 O rows (every 64-column chunk) before one set of
// TMA stores, so no chunk waits for the previous chunk's store to read the slot (+1.5..2% on
// the short-unit pack_tail config, neutral elsewhere). 0: one 64-column chunk slot per warp,
// reused chunk by chunk.
#define FA2_STG_FULL 1
#endif
#ifndef FA2_L2_HINTS
#define FA2_L2_HINTS 1  // 1: K/V loads evict_last, Q loads evict_first in L2; 0: evict_normal for both
#endif
#ifndef FA2_TWO_ISSUERS
// 1: (no split-KV pairs) warp 8 issues Q tile 0's MMAs and warp 10 tile 1's, so one tile's
// hand-offs are not served after the other tile's MMA issue. 0 (shipped): warp 8 issues both,
// whole GEMMs in the order PV(0) QK(0) PV(1) QK(1). Measured: two issuers 16-19% slower on every
// config (the tensor pipe then interleaves the two tiles' MMAs); kept as an ablation alternative.
#define FA2_TWO_ISSUERS 0
#endif
#ifndef FA2_PERSISTENT
#define FA2_PERSISTENT 1  // 0: one CTA per work unit (the grid covers the units) without split-KV too
#endif
#ifndef FA2_DEFER_EPI
// 1: a softmax warp writes a unit's output during the next unit's first step, after that step's
// P hand-off (where it would otherwise wait for the next S), instead of between the units; the
// next unit's first PV, which overwrites O_t, waits on O_EMPTY until O_t is in registers.
// Measured 1-3.4% slower (headline, MHA causal, pack_tail; same box, with or without the branch
// marked cold), like moving the epilogue to warps of its own. 0 (shipped): the epilogue runs
// when the unit ends.
#define FA2_DEFER_EPI 0
#endif
#ifndef FA2_SEP_P_D64
// 1: at D = 64 (outside split-KV) P_t gets its own 64 TMEM columns (S 0-255, O 256-383, P 384-511)
// instead of overwriting the upper half of S_t, so the next QK of a tile is issued as soon as its
// softmax warps have loaded S_t, not after the PV that reads P. Measured 9-12% slower (D = 64 fp16
// and bf16, causal and not): before rewriting P_t a softmax warp must now wait for the previous
// PV, which queues behind the other tile's GEMMs, where S_t(j + 1) arriving used to imply it.
// 0 (shipped): P overwrites S_t, as at D = 128 (which has no TMEM left for a separate P).
#define FA2_SEP_P_D64 0
#endif
#ifndef FA2_PAIR
// 1: fixed-length D = 128 launches without split-KV of at least FA2_PAIR_MIN_ROWS packed rows per
// (batch, head block) run on CTA pairs (fa2_pair_sm100.cuh: one M = 256 cta_group::2 MMA over two
// SMs, K/V split between them). Same-box A/B against the single-CTA kernel: headline +0.5..2.4%,
// pack_tail +3..5%, mha_causal -4.5..6%, MQA -1.7%, non-causal D = 128 within +-2%. Each SM then
// moves half the K/V bytes and its MMAs run at ~64 instead of ~75-80 cycles per k-step, but every
// hand-off waits for the slower of two SMs and the even CTA's MMA warp still slows the softmax
// warp on its SMSP. 0 (shipped): always the single-CTA kernel.
#define FA2_PAIR 0
#endif
#ifndef FA2_PAIR_MIN_ROWS
#define FA2_PAIR_MIN_ROWS 1024
#endif
#ifndef FA2_TRACE
// 1: compile the step-timing stamps (see FA2_STAMP); 0 (shipped): none.
#define FA2_TRACE 0
#endif
#ifndef FA2_WARP_WAIT_D128
// 1 (shipped): at D = 128 the softmax warps wait for S and O with warp-voted probes
// (mbar_wait_warp: uniform branches instead of a per-lane probe loop and one vote at the end).
// Same-box A/B, two runs: headline +0.2/+0.5%, mha_causal 0/+1.1%, pack_tail +0.6/+0.6%; at
// D = 64 (full_long) -0.9/-2.0%, so the D = 64 build keeps the per-lane loop.
#define FA2_WARP_WAIT_D128 1
#endif
#ifndef FA2_HEAD_MAJOR
// 1: without a causal mask the persistent CTAs walk the units (batch, head) slice by slice;
// 0: row block by row block, as with a causal mask (every head's K/V in flight at once).
#define FA2_HEAD_MAJOR 1
#endif
#ifndef FA2_SEQ_EXP
// 1: the two softmax warps of a lane quadrant (tile 0 and tile 1, on the same SMSP) take turns
// on the exponential phase of a step (tile 0 step j, tile 1 step j, tile 0 step j + 1, ...)
// through a bounded mbarrier hand-shake, so they never compete for the MUFU and issue slots.
// The loads and row max of one overlap the other's exponentials. 0: no ordering.
#define FA2_SEQ_EXP 0
#endif
#ifndef FA2_FFMA_PASS
// 1: x = s * qk_scale - m is computed for the whole row in one pass of packed FMAs before the
// exponentials (no dependency between them); 0: fused into the per-chunk exponential loop.
#define FA2_FFMA_PASS 0
#endif
template <int D>
__host__ __device__ constexpr bool spec_max() {
  return D == 128 ? FA2_SPEC_MAX_D128 != 0 : FA2_SPEC_MAX_D64 != 0;
}
template <int D, bool BF16>
__host__ __device__ constexpr uint32_t emu_pair_mask() {
  return D == 128 ? static_cast<uint32_t>(FA2_EMU_MASK_D128)
                  : (BF16 ? static_cast<uint32_t>(FA2_EMU_MASK_D64_BF16) : static_cast<uint32_t>(FA2_EMU_MASK_D64));
}
constexpr int P_SPLIT = FA2_P_SPLIT;
static_assert(P_SPLIT >= 1 && P_SPLIT <= 3, "P hand-off split");
constexpr int NCH = SCOLS / 32;                          // 32-score chunks per softmax warp
constexpr int P_SPLIT_W = HALVES == 1 ? P_SPLIT : 1;     // of them, handed over before the rest
// TMEM columns of S_t, per warp: its SCOLS scores at t * BN + h * SCOLS. P (2 per column)
// overwrites the upper half of that range; with HALVES == 2 the lowest column, read into
// registers like the rest, then carries the warp's row max to the other warp of the row.
constexpr int P_OFF = SCOLS / 2;
// setmaxnreg draws on the registers the CTA was launched with (threads x REGS_LAUNCH).
template <int D>
constexpr bool regs_fit() {
  return SOFTMAX_WARPS * regs_softmax<D>() + (NUM_WARPS - SOFTMAX_WARPS) * regs_other<D>() <= NUM_WARPS * REGS_LAUNCH &&
         regs_other<D>() >= 24 && regs_softmax<D>() % 8 == 0 && regs_softmax<D>() <= 256;
}
static_assert(regs_fit<128>() && regs_fit<64>(), "register split exceeds the launch budget");
static_assert(NUM_THREADS * REGS_LAUNCH <= 65536, "launch register budget");
static_assert(HALVES == 1 || !FA2_TWO_ISSUERS, "two MMA issuers need the 12-warp layout");
static_assert(HALVES == 1 || !FA2_SEQ_EXP, "the exponential hand-shake needs the 12-warp layout");

// Shared-memory layout of one CTA. SPLIT: the split-KV build, which writes fp32 partials from
// registers (no O staging) and, streaming K/V from HBM, uses a deeper ring.
template <int D, bool SPLIT = false>
struct Cfg {
  static_assert(D == 64 || D == 128, "compiled head dims");
  static constexpr int CHUNKS = D / 64;             // 64-element (128-byte) swizzle atoms along d
  static constexpr int CHUNK_BYTES = 128 * 128;     // 128 rows x 128 bytes
  static constexpr int TILE_BYTES = BN * D * 2;     // == BM * D * 2
  // K/V ring depth (K_j and V_j take one slot each)
  static constexpr int STAGES = SPLIT ? ((D == 128) ? 4 : 8) : ((D == 128) ? FA2_STAGES_D128 : FA2_STAGES_D64);
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_KV = Q_TILES * TILE_BYTES;
  // Epilogue: each epilogue warp writes EPI_COLS columns of O for its 32 rows. With two
  // warps per row, D = 128 gives each 64 columns; at D = 64 the first warp of the row
  // writes all of them.
  static constexpr int EPI_COLS = (HALVES == 2 && D == 128) ? 64 : D;
  static constexpr int EPI_WARPS = (EPI_COLS * HALVES == D) ? SOFTMAX_WARPS : 8;
  // O staging for the TMA store: slots of 32 rows x 64 columns (128-byte swizzle, the
  // O tensor map's box) per epilogue warp.
  static constexpr int STG_SLOT_BYTES = 32 * 128;                        // one 64-column chunk
  static constexpr int STG_WARP_BYTES = SPLIT ? 0 : (FA2_STG_FULL ? EPI_COLS / 64 : 1) * STG_SLOT_BYTES;
  static constexpr int OFF_STG = OFF_KV + STAGES * TILE_BYTES;
  static constexpr int OFF_BAR = OFF_STG + EPI_WARPS * STG_WARP_BYTES;
  // barrier slots
  static constexpr int B_Q = 0;                     // [2]  Q tile landed
  static constexpr int B_KV_FULL = 2;               // [S]  K/V tile landed
  static constexpr int B_KV_EMPTY = 2 + STAGES;     // [S]  K/V slot released by the MMAs
  static constexpr int B_S_FULL = 2 + 2 * STAGES;   // [2]  S_t in TMEM
  static constexpr int B_P_FULL = 4 + 2 * STAGES;   // [2]  P_t columns [0, 32*P_SPLIT) in TMEM, O_t rescaled
  static constexpr int B_O_FULL = 6 + 2 * STAGES;   // [2]  last PV of tile t retired
  static constexpr int B_MMA_DONE = 8 + 2 * STAGES; // [1]  every MMA retired (teardown)
  static constexpr int B_P_LATE = 9 + 2 * STAGES;   // [2]  the remaining P_t columns in TMEM
  static constexpr int B_Q_EMPTY = 11 + 2 * STAGES; // [2]  last QK of tile t of a unit retired: Q_t reloadable
  static constexpr int B_XCH = 13 + 2 * STAGES;     // [8]  (HALVES == 2) row-pair exchange of tile t, quadrant q
  static constexpr int B_SEQ = 13 + 2 * STAGES;     // [8]  (FA2_SEQ_EXP) exponential phase of tile t, quadrant q done
  static constexpr int B_S_EMPTY = 21 + 2 * STAGES; // [2]  (SEP_P) S_t read by the softmax warps: the next QK may write it
  static constexpr int B_P_EMPTY = 23 + 2 * STAGES; // [2]  (SEP_P) PV(t) retired: P_t may be rewritten, O_t rescaled
  static constexpr int B_O_EMPTY = 25 + 2 * STAGES; // [2]  (DEFER) O_t of the previous unit in registers: PV may overwrite it
  static constexpr int NUM_BARS = 27 + 2 * STAGES;
  // P_t in TMEM columns of its own (see FA2_SEP_P_D64), for the fixed-length D = 64 build.
  static constexpr bool SEP_P = D == 64 && !SPLIT && HALVES == 1 && !FA2_TWO_ISSUERS && FA2_SEP_P_D64 != 0;
  // Deferred epilogue (FA2_DEFER_EPI) for the persistent single-issuer layout.
  static constexpr bool DEFER = FA2_DEFER_EPI != 0 && !SPLIT && HALVES == 1 && !FA2_TWO_ISSUERS && !SEP_P;
  static constexpr int OFF_TMEM_PTR = OFF_BAR + NUM_BARS * 8;
  static constexpr int SMEM_BYTES = OFF_TMEM_PTR + 16;
  static constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;  // slack to align the base to 1024 B
  static constexpr int TMEM_O = 2 * BN;                 // O_t at TMEM_O + t * D
  static constexpr int TMEM_P = TMEM_O + 2 * D;         // SEP_P: P_t at TMEM_P + t * BN / 2
  static_assert(TMEM_O + 2 * D + (SEP_P ? BN : 0) <= TMEM_COLS, "TMEM budget");
  // HALVES == 2: column that carries warp h's row sum to the other warp of the row in the
  // epilogue. D = 128: the first of its own O columns (read before it is overwritten);
  // D = 64: spare columns past O_1.
  __device__ static constexpr int tmem_lx(int t, int h) {
    return D == 128 ? TMEM_O + t * D + h * 64 : TMEM_O + 2 * D + t * 2 + h;
  }
  static_assert(SMEM_ALLOC <= 227 * 1024, "shared memory budget");
};

// Division of 0 <= n < 2^31 by a divisor d >= 1 fixed at launch, as a multiply-high, an add
// and a shift (Granlund & Montgomery, "Division by invariant integers using multiplication",
// PLDI 1994): with l = ceil(log2 d) and m = floor(2^32 (2^l - d) / d) + 1,
// n / d == (umulhi(n, m) + n) >> l. Unit decoding runs between a unit's last softmax step
// and the next unit's first one, where a hardware-free division chain is on the critical path.
struct FastDiv {
  uint32_t d, m, l;
  __host__ __device__ __forceinline__ uint32_t div(uint32_t n) const { return (__umulhi_hd(n, m) + n) >> l; }
  __host__ __device__ __forceinline__ static uint32_t __umulhi_hd(uint32_t a, uint32_t b) {
#ifdef __CUDA_ARCH__
    return __umulhi(a, b);
#else
    return static_cast<uint32_t>((static_cast<uint64_t>(a) * b) >> 32);
#endif
  }
};

inline FastDiv make_fastdiv(uint32_t d) {
  FastDiv f;
  f.d = d;
  f.l = 0;
  while ((1ull << f.l) < d) ++f.l;
  f.m = static_cast<uint32_t>(((1ull << 32) * ((1ull << f.l) - d)) / d + 1ull);
  return f;
}

struct KArgs {
  int n_q, n_kv, group, pack, hblocks;  // hblocks = H_q / pack
  // Causal: query position i sees key columns c <= i + causal_off. 0 is the reference's
  // top-left alignment (N_q == N_kv); N_kv - N_q aligns the last query with the last key
  // (bottom-right, for chunked prefill and decode with N_q <= N_kv).
  int causal_off;
  int bottom_right;                     // variable-length: causal_off is N_kv - N_q per sequence
  // Variable-length batch: sequence b owns Q positions [cu_q[b], cu_q[b + 1]) and K/V positions
  // [cu_kv[b], cu_kv[b + 1]) of one packed token axis (the tensor maps' b extent is 1); n_q and
  // n_kv are the largest lengths. nullptr: fixed lengths n_q / n_kv, batch on the maps' b axis.
  const int* cu_q;
  const int* cu_kv;
  // Paged K/V: sequence b's key j lives in page block_table[b * bt_stride + j / page_size], row
  // j % page_size (the K/V tensor maps' b axis is the page, n the row); seqlens_kv[b] keys.
  const int* block_table;
  const int* seqlens_kv;
  int bt_stride, page_size;
  void* o;                              // output base and element strides (h, n): used for the
  int64_t oh, on;                       // rows of a variable-length sequence's last O box
  // Columns of the caller's head dimension (16 or 32 on the D = 64 build, else D). The tensor
  // maps have this extent, so TMA loads fill the columns past it with zeros (they add nothing to
  // Q K^T and make zero O columns) and TMA stores clip them; register stores check it.
  int d_real;
  int pack_shift;                       // pack == 1 << pack_shift (pack divides 128)
  FastDiv div_xblocks, div_hblocks, div_group, div_mblocks;
  float qk_scale;
  int* err;
  const int* gate;
  long long timeout;
  // Work units: (256-row block mb, batch x head block x), xblocks * mblocks of them.
  // persistent != 0 (no split-KV): gridDim.x CTAs, one per SM, walk the units in the order
  // u = mi * xblocks + x with mi = 0 the heaviest causal block; CTA c takes u = n * G + c in
  // even rounds n and u = n * G + (G - 1 - c) in odd ones (a snake, so each CTA gets a similar
  // mix of long and short causal blocks). Otherwise the grid is (xblocks, mblocks, splits) and
  // each CTA does the one unit of its block index.
  int persistent, xblocks, mblocks, num_units;
  // split-KV: CTA (x, y, z) covers K/V tiles [z * split_tiles, (z + 1) * split_tiles) of its
  // range and writes fp32 O / l plus the row log2-sum-exp to the workspace (num_splits > 1).
  int num_splits, split_tiles, rows_pad;
  // dual split (num_splits > 1, non-causal, all rows in Q tile 0): both Q-tile slots use the
  // same 128 query rows, tile t walking split 2z + t, so a CTA streams two K/V ranges at once.
  int dual;
  float* o_part;    // [num_splits][gridDim.x][rows_pad][D]
  float* lse_part;  // [num_splits][gridDim.x][rows_pad]
};

// K/V tiles a CTA of 256-row block mb visits (>= 1): its causal band end, or all of N_kv.
// pack == 1 << pack_shift; causal_off >= 0 is the bottom-right shift (KArgs::causal_off).
template <bool CAUSAL>
__host__ __device__ __forceinline__ int cta_kv_tiles(int mb, int n_q, int n_kv, int pack_shift, int causal_off) {
  int kv_end = n_kv;
  if (CAUSAL) {
    const int last_pos = min((mb * 256 + 255) >> pack_shift, n_q - 1);
    kv_end = min(last_pos + 1 + causal_off, n_kv);
  }
  return (kv_end + 127) / 128;
}

// One work unit: packed Q rows [row0, row0 + 256) of batch b, q heads from hq0 (K/V head hkv),
// against K/V tiles [j0, j0 + J) (in dual mode the second Q-tile slot walks [j0b, j0b + J)).
// q0 / kv0: first Q / K/V position of the unit's sequence on the tensor maps' n axis, tb / tbkv
// the Q/O and K/V maps' b coordinate (0 for a packed token axis; paged K/V take their page per
// tile); n_q / n_kv / coff: the sequence's lengths and causal shift.
struct Unit {
  int x, b, hq0, hkv, row0, j0, j0b, J;
  int q0, kv0, tb, tbkv, n_q, n_kv, coff;
  int J0;  // CTA pairs: K/V tiles of the unit's first 256 rows (<= J, which covers all 512)
};

// Unit slot n of this CTA; false when the CTA has no n-th slot. J == 0: the unit is empty (a
// split past its row block's causal band, or a row block past a shorter sequence's end).
// VARLEN: the variable-length build (a.cu_q != nullptr exactly then).
template <bool CAUSAL, bool VARLEN>
__device__ __forceinline__ bool get_unit(const KArgs& a, int n, Unit& u) {
  int mb, z = 0;
  if (a.persistent) {
    // n * G + c < num_units + G < 2^32: 32-bit unsigned arithmetic is exact.
    const uint32_t G = gridDim.x, c = blockIdx.x, nn = static_cast<uint32_t>(n);
    const uint32_t idx = nn * G + ((nn & 1u) ? (G - 1u - c) : c);
    if (idx >= static_cast<uint32_t>(a.num_units)) return false;
    if (CAUSAL || !FA2_HEAD_MAJOR) {
      // Row-block major, heaviest causal block first: the CTAs of a round share a row block
      // and span the (batch, head) slices, which keeps the longest units at the front.
      const uint32_t mi = a.div_xblocks.div(idx);
      u.x = static_cast<int>(idx - mi * a.div_xblocks.d);
      mb = CAUSAL ? a.mblocks - 1 - static_cast<int>(mi) : static_cast<int>(mi);
    } else {
      // Without a causal mask every unit has the same length: slice major, so the CTAs of a
      // round read the K/V of a few heads (it stays in L2) instead of one row block of every head.
      const uint32_t xs = a.div_mblocks.div(idx);
      u.x = static_cast<int>(xs);
      mb = static_cast<int>(idx - xs * a.div_mblocks.d);
    }
  } else {
    if (n > 0) return false;
    u.x = static_cast<int>(blockIdx.x);
    mb = CAUSAL ? static_cast<int>(gridDim.y - 1 - blockIdx.y) : static_cast<int>(blockIdx.y);
    z = static_cast<int>(blockIdx.z);
  }
  u.b = static_cast<int>(a.div_hblocks.div(static_cast<uint32_t>(u.x)));
  u.hq0 = (u.x - u.b * a.hblocks) << a.pack_shift;
  u.hkv = static_cast<int>(a.div_group.div(static_cast<uint32_t>(u.hq0)));
  static_assert(Q_TILES * BM == 256 && BN == 128, "cta_kv_tiles assumes 256-row CTAs, 128-row K/V tiles");
  u.row0 = mb * (Q_TILES * BM);
  u.j0 = 0;
  u.j0b = 0;
  if constexpr (VARLEN) {
    // Per-sequence lengths: queries packed by cu_q or fixed; keys packed by cu_kv, counted by
    // seqlens_kv (paged K/V) or fixed.
    if (a.cu_q != nullptr) {
      u.q0 = __ldg(a.cu_q + u.b);
      u.n_q = __ldg(a.cu_q + u.b + 1) - u.q0;
      u.tb = 0;
    } else {
      u.q0 = 0;
      u.n_q = a.n_q;
      u.tb = u.b;
    }
    if (a.cu_kv != nullptr) {
      u.kv0 = __ldg(a.cu_kv + u.b);
      u.n_kv = __ldg(a.cu_kv + u.b + 1) - u.kv0;
      u.tbkv = 0;
    } else {
      u.kv0 = 0;
      u.n_kv = a.seqlens_kv != nullptr ? __ldg(a.seqlens_kv + u.b) : a.n_kv;
      u.tbkv = u.b;
    }
    u.coff = a.bottom_right ? u.n_kv - u.n_q : 0;
    if (u.n_q < 0 || u.n_kv < 0 || u.n_q > a.n_q || u.n_kv > a.n_kv) {
      // Lengths the launch was not sized for: reported, and the unit is left out.
      if (a.err != nullptr) atomicCAS(a.err, 0, FA2_ERR_SHAPE);
      u.J = 0;
      return true;
    }
    if (u.row0 >= (u.n_q << a.pack_shift)) {  // past this sequence's last row
      u.J = 0;
      return true;
    }
  } else {
    u.q0 = 0;
    u.kv0 = 0;
    u.tb = u.b;
    u.tbkv = u.b;
    u.n_q = a.n_q;
    u.n_kv = a.n_kv;
    u.coff = a.causal_off;
  }
  // At least one K/V tile: rows that see no key at all (a sequence without keys, or
  // bottom-right rows before the first key) then get exact zeros from a fully masked tile.
  const int J_cta = max(1, cta_kv_tiles<CAUSAL>(mb, u.n_q, u.n_kv, a.pack_shift, u.coff));
  u.J = J_cta;
  if (a.num_splits > 1) {
    if (a.dual) {
      u.j0 = 2 * z * a.split_tiles;
      u.j0b = u.j0 + a.split_tiles;
      u.J = (u.j0 < J_cta) ? a.split_tiles : 0;  // tiles past N_kv load as zeros and are masked
    } else {
      u.j0 = z * a.split_tiles;
      u.J = max(0, min(J_cta - u.j0, a.split_tiles));
    }
  }
  return true;
}

// The next non-empty unit after slot `slot` (which it advances past the unit); false when the
// CTA has no more. Every role walks the same slots, so all of them see the same units.
template <bool CAUSAL, bool VARLEN>
__device__ __forceinline__ bool next_unit(const KArgs& a, int& slot, Unit& u) {
  while (get_unit<CAUSAL, VARLEN>(a, slot, u)) {
    ++slot;
    if (u.J > 0) return true;
  }
  return false;
}

// Paged K/V: page indices of one sequence's block-table row for the TMA producer. Holds the page
// slot in use and the one after it; looking up a new slot starts the load of the next entry, which
// is used (and waited for) only when the producer reaches that slot.
struct PageCache {
  int cur_pi, cur_page, next_pi, next_page;
  __device__ __forceinline__ void reset() { cur_pi = next_pi = -1; }
  // Page of slot pi of `bt`, or -1 (loads zeros) for slots past the sequence's last page.
  __device__ __forceinline__ int page(const int* bt, int pi, int pages_used) {
    if (pi >= pages_used) return -1;
    if (pi != cur_pi) {
      if (pi == next_pi) {
        cur_page = next_page;
      } else {
        cur_page = __ldg(bt + pi);
      }
      cur_pi = pi;
      next_pi = pi + 1;
      next_page = next_pi < pages_used ? __ldg(bt + next_pi) : -1;
    }
    return cur_page;
  }
};

// ---------------------------------------------------------------- softmax helpers

// Max of 64 scores (two 32-column chunks) with four independent 3-input max chains.
__device__ __forceinline__ float row_max64(const uint32_t (&s0)[32], const uint32_t (&s1)[32]) {
  float m0 = -INFINITY, m1 = -INFINITY, m2 = -INFINITY, m3 = -INFINITY;
#pragma unroll
  for (int i = 0; i < 32; i += 4) {
    m0 = fmax3(m0, __uint_as_float(s0[i + 0]), __uint_as_float(s0[i + 1]));
    m1 = fmax3(m1, __uint_as_float(s0[i + 2]), __uint_as_float(s0[i + 3]));
    m2 = fmax3(m2, __uint_as_float(s1[i + 0]), __uint_as_float(s1[i + 1]));
    m3 = fmax3(m3, __uint_as_float(s1[i + 2]), __uint_as_float(s1[i + 3]));
  }
  return fmax3(fmaxf(m0, m1), m2, m3);
}

// Max of a warp's scores of its row: 128 (four chunks) or 64 (two).
template <int N>
__device__ __forceinline__ float row_max_chunks(const uint32_t (&s)[N][32]) {
  static_assert(N == 2 || N == 4, "chunks per softmax warp");
  if constexpr (N == 4) {
    return fmaxf(row_max64(s[0], s[1]), row_max64(s[2], s[3]));
  } else {
    return row_max64(s[0], s[1]);
  }
}

// Scores of columns c0 + i with c0 + i > lim are set to -inf (causal / end-of-sequence mask).
__device__ __forceinline__ void mask_chunk(uint32_t (&s)[32], int c0, int lim) {
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    if (c0 + i > lim) s[i] = __float_as_uint(-INFINITY);
  }
}

// p = exp2(s * scale - m) for 32 scores: packed to 16 words of (lo, hi) halves for the PV
// GEMM, and written back into s as fp32 for the row sum. The pairs set in EMU_MASK are
// computed on the FMA pipe (exp2_poly_x2); the subset depends only on the column index.
template <bool BF16, uint32_t EMU_MASK, bool PRESCALED = false>
__device__ __forceinline__ void make_p32(uint32_t (&s)[32], uint64_t sc2, uint64_t nm2, uint32_t (&pk)[16]) {
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    const uint64_t s2 = f2_pack(__uint_as_float(s[2 * e]), __uint_as_float(s[2 * e + 1]));
    const uint64_t x2 = PRESCALED ? s2 : f2_fma(s2, sc2, nm2);
    float x0, x1, p0, p1;
    f2_unpack(x2, x0, x1);
    if ((EMU_MASK >> e) & 1u) {
      exp2_poly_x2<BF16 ? 3 : FA2_POLY_DEG_FP16>(x0, x1, p0, p1);
    } else {
      p0 = ex2_mufu(x0);
      p1 = ex2_mufu(x1);
    }
    pk[e] = cvt_pack2<BF16>(p0, p1);
    s[2 * e] = __float_as_uint(p0);
    s[2 * e + 1] = __float_as_uint(p1);
  }
}

// As make_p32, but s keeps the scores (a redo may need them) and the fp32 p are added into the
// row-sum accumulators instead: pair e goes to acc2[e % 4], the order make_p32's caller sums in.
template <bool BF16, uint32_t EMU_MASK>
__device__ __forceinline__ void make_p32_sum(const uint32_t (&s)[32], uint64_t sc2, uint64_t nm2, uint32_t (&pk)[16],
                                             uint64_t (&acc2)[4]) {
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    const uint64_t x2 = f2_fma(f2_pack(__uint_as_float(s[2 * e]), __uint_as_float(s[2 * e + 1])), sc2, nm2);
    float x0, x1, p0, p1;
    f2_unpack(x2, x0, x1);
    if ((EMU_MASK >> e) & 1u) {
      exp2_poly_x2<BF16 ? 3 : FA2_POLY_DEG_FP16>(x0, x1, p0, p1);
    } else {
      p0 = ex2_mufu(x0);
      p1 = ex2_mufu(x1);
    }
    pk[e] = cvt_pack2<BF16>(p0, p1);
    acc2[e & 3] = f2_add(acc2[e & 3], f2_pack(p0, p1));
  }
}

// O row *= alpha for this thread's NCOL columns of O_t (its TMEM lane), 16 at a time.
template <int NCOL>
__device__ __forceinline__ void rescale_o_cols(uint32_t tO, float alpha) {
  const uint64_t a2 = f2_pack(alpha, alpha);
#pragma unroll 1  // rare path: kept rolled, which keeps the unmasked step free of spills
  for (int c = 0; c < NCOL / 16; ++c) {
    uint32_t o[16];
    tmem_ld16(tO + c * 16, o);
    tmem_wait_ld();
    reg_fence16(o);
#pragma unroll
    for (int i = 0; i < 16; i += 2) {
      float x, y;
      f2_unpack(f2_mul(f2_pack(__uint_as_float(o[i]), __uint_as_float(o[i + 1])), a2), x, y);
      o[i] = __float_as_uint(x);
      o[i + 1] = __float_as_uint(y);
    }
    tmem_st16(tO + c * 16, o);
  }
  tmem_wait_st();
}

// Every lane waits for `bar`'s phase; true when it completed for the whole warp.
__device__ __forceinline__ bool warp_wait_pv(uint32_t bar, uint32_t parity, const KArgs& a) {
  const bool w = mbar_wait(bar, parity, a.timeout, a.err);
  return __all_sync(0xffffffffu, w);
}

// Step timing (FA2_TRACE=1 builds only; triton-fa2-forward_b200/step_trace.py reads it): SM-clock
// stamps of CTA 0's first FA2_TRACE_UNITS units, per K/V step j and Q tile t, at the hand-off points
// of the softmax warps (warp q == 0 of each tile; per-warp copies at 16 + q ...) and the MMA thread.
// A stamp is a clock64 read and one global store; nothing is skipped or reordered.
#if FA2_TRACE
#define FA2_TRACE_UNITS 4
#define FA2_TRACE_STEPS 80
__device__ long long g_fa2_trace[FA2_TRACE_UNITS][FA2_TRACE_STEPS][2][32];
#define FA2_STAMP(n_, j_, t_, e_)                                                           \
  do {                                                                                      \
    if (blockIdx.x == 0 && (n_) < FA2_TRACE_UNITS && (j_) < FA2_TRACE_STEPS)                \
      g_fa2_trace[(n_)][(j_)][(t_)][(e_)] = clock64();                                      \
  } while (0)
#else
#define FA2_STAMP(n_, j_, t_, e_) \
  do {                            \
  } while (0)
#endif

// ------------------------------------------------------------------------ kernel
// SPLIT: the split-KV build (num_splits > 1); VARLEN: the variable-length build
// (cu_seqlens given). The host launches each exactly then; never both.
template <int D, bool CAUSAL, bool BF16, bool SPLIT, bool VARLEN>
__global__ void __launch_bounds__(NUM_THREADS, 1)
fa2_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
               const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
               const KArgs a) {
  using C = Cfg<D, SPLIT>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t sraw = smem_u32(smem_raw);
  const uint32_t sbase = (sraw + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (sbase - sraw);
  auto bar = [&](int i) -> uint32_t { return sbase + C::OFF_BAR + 8u * static_cast<uint32_t>(i); };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Dual mode exists only with split-KV, which is never persistent: one unit per CTA.
  const bool dual = (a.dual != 0);
  {
    Unit u0;
    int s0 = 0;
    if (!next_unit<CAUSAL, VARLEN>(a, s0, u0)) return;  // nothing to do (uniform, before any sync)
  }

  // MMA-issuing threads: every K/V slot is released, and the teardown barrier arrived at, by each.
  const uint32_t issuers = (FA2_TWO_ISSUERS && !dual) ? 2u : 1u;
  if (warp == LOAD_WARP && lane == 0) {
    for (int t = 0; t < 2; ++t) {
      mbar_init(bar(C::B_Q + t), 1);
      mbar_init(bar(C::B_Q_EMPTY + t), 1);
      mbar_init(bar(C::B_S_FULL + t), 1);
      mbar_init(bar(C::B_P_FULL + t), BM * HALVES);
      mbar_init(bar(C::B_P_LATE + t), BM * HALVES);
      mbar_init(bar(C::B_O_FULL + t), 1);
    }
    if constexpr (HALVES == 2) {
      for (int x = 0; x < 8; ++x) mbar_init(bar(C::B_XCH + x), 64);
    }
    if constexpr (FA2_SEQ_EXP != 0) {
      for (int x = 0; x < 8; ++x) mbar_init(bar(C::B_SEQ + x), 32);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(bar(C::B_S_EMPTY + t), BM);  // every softmax thread of the tile
      mbar_init(bar(C::B_P_EMPTY + t), 1);   // the MMA thread's commit
      mbar_init(bar(C::B_O_EMPTY + t), BM);  // every softmax thread of the tile
    }
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(bar(C::B_KV_FULL + s), 1);
      mbar_init(bar(C::B_KV_EMPTY + s), issuers);
    }
    mbar_init(bar(C::B_MMA_DONE), issuers);
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  if (warp == MMA_WARP) {
    __syncwarp();
    tmem_alloc(sbase + C::OFF_TMEM_PTR, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + C::OFF_TMEM_PTR);

  bool ok = true;

  if (warp == LOAD_WARP) {
    reg_dealloc<regs_other<D>()>();
    // ------------------------------------------------------------- TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmO);
      // K/V are re-read by every Q block of their head, Q is read once.
      const uint64_t pol_kv = FA2_L2_HINTS ? l2_policy_evict_last() : l2_policy_evict_normal();
      const uint64_t pol_q = FA2_L2_HINTS ? l2_policy_evict_first() : l2_policy_evict_normal();
      int q_loads0 = 0, q_loads1 = 0;
      auto load_q = [&](const Unit& u, int t) {
        const int R = u.row0 + t * BM;
        const int pos = R >> a.pack_shift;
        const int h = u.hq0 + (R & (a.pack - 1));
        mbar_arrive_expect_tx(bar(C::B_Q + t), C::TILE_BYTES);
#pragma unroll
        for (int c = 0; c < C::CHUNKS; ++c) {
          tma_load_4d(sbase + C::OFF_Q + t * C::TILE_BYTES + c * C::CHUNK_BYTES, &tmQ, bar(C::B_Q + t),
                      c * 64, h, u.q0 + pos, u.tb, pol_q);
        }
        if (t == 0) ++q_loads0; else ++q_loads1;
      };
      // Optional start gate: no load is issued before *gate != 0 (bounded like every wait).
      if (a.gate != nullptr) ok = flag_wait(a.gate, a.timeout, a.err);
      int i = 0;  // K/V tiles issued into the ring, over all units
      int slot = 0;
      PageCache page_a, page_b;  // two K/V streams in dual mode; named, so they stay in registers
      for (int n = 0; ok; ++n) {
        Unit u;
        if (!next_unit<CAUSAL, VARLEN>(a, slot, u)) break;
        page_a.reset();
        page_b.reset();
        // Q_t's buffer is free once the last QK GEMM of tile t of the previous unit retired.
        if (n > 0 && !mbar_wait(bar(C::B_Q_EMPTY + 0), static_cast<uint32_t>(n - 1) & 1u, a.timeout, a.err)) {
          ok = false;
          break;
        }
        load_q(u, 0);
        // Ring order == the MMA warp's consumption order. Normal: K0, V0, K1, V1, ... (each
        // tile feeds both Q tiles; the next unit's K0 follows this unit's last V). Dual: Ka0,
        // Kb0, then per step j: Va_j, Ka_j+1, Vb_j, Kb_j+1.
        const int n_tiles = dual ? 4 * u.J : 2 * u.J;
        for (int k = 0; k < n_tiles; ++k) {
          const int st = i % C::STAGES;
          const uint32_t ph = static_cast<uint32_t>(i / C::STAGES) & 1u;
          if (!mbar_wait(bar(C::B_KV_EMPTY + st), ph ^ 1u, a.timeout, a.err)) {
            ok = false;
            break;
          }
          bool is_v;
          int kv_tile;
          if (!dual) {
            is_v = (k & 1) != 0;
            kv_tile = u.j0 + (k >> 1);
          } else if (k < 2) {
            is_v = false;
            kv_tile = (k == 0) ? u.j0 : u.j0b;
          } else {
            const int g = (k - 2) >> 2, rr = (k - 2) & 3;
            if (g == u.J - 1) {  // last step: Va, Vb
              is_v = true;
              kv_tile = (rr == 0 ? u.j0 : u.j0b) + g;
            } else {
              is_v = (rr & 1) == 0;
              kv_tile = (rr < 2 ? u.j0 : u.j0b) + g + (is_v ? 0 : 1);
            }
          }
          mbar_arrive_expect_tx(bar(C::B_KV_FULL + st), C::TILE_BYTES);
          const CUtensorMap* m = is_v ? &tmV : &tmK;
          const uint32_t dst = sbase + C::OFF_KV + st * C::TILE_BYTES;
          if (VARLEN && a.block_table != nullptr) {
            // Paged K/V: the tile's 128 keys are one page slice (page_size >= 128) or
            // 128 / page_size whole pages, each a box of page_size rows at its row offset in the
            // slot (a multiple of 8 rows, so the 128-byte swizzle lines up). Page slots past the
            // sequence's last page are not read from the table: coordinate -1 loads zeros.
            const int* bt = a.block_table + static_cast<int64_t>(u.b) * a.bt_stride;
            const int pos = kv_tile * BN;
            const int pages_used = (u.n_kv + a.page_size - 1) / a.page_size;
            const int boxes = a.page_size >= BN ? 1 : BN / a.page_size;
            // Page lookups go through a small cache per K/V stream (two in dual mode): the page
            // in use and the table entry after it, fetched as soon as the current one is known,
            // so its load overlaps the ring waits instead of stalling the next tile's issue.
            const bool stream_b = dual && kv_tile >= u.j0b;
            for (int sub = 0; sub < boxes; ++sub) {
              const int pi = pos / a.page_size + sub;
              const int page = stream_b ? page_b.page(bt, pi, pages_used) : page_a.page(bt, pi, pages_used);
              const int row = a.page_size >= BN ? pos % a.page_size : 0;
#pragma unroll
              for (int c = 0; c < C::CHUNKS; ++c) {
                tma_load_4d(dst + c * C::CHUNK_BYTES + sub * a.page_size * 128, m, bar(C::B_KV_FULL + st), c * 64,
                            row, u.hkv, page, pol_kv);
              }
            }
          } else {
#pragma unroll
            for (int c = 0; c < C::CHUNKS; ++c) {
              tma_load_4d(dst + c * C::CHUNK_BYTES, m, bar(C::B_KV_FULL + st), c * 64, u.kv0 + kv_tile * BN, u.hkv,
                          u.tbkv, pol_kv);
            }
          }
          ++i;
          if (k == 0 && !dual) {
            if (n > 0 &&
                !mbar_wait(bar(C::B_Q_EMPTY + 1), static_cast<uint32_t>(n - 1) & 1u, a.timeout, a.err)) {
              ok = false;
              break;
            }
            load_q(u, 1);
          }
        }
      }
      // Drain: every TMA write into this CTA's shared memory must land before the CTA
      // can exit, also when another role gave up early. Loads older than the last STAGES
      // were consumed (their slots were refilled), so they have landed.
      for (int d = max(0, i - C::STAGES); d < i; ++d) {
        mbar_wait(bar(C::B_KV_FULL + d % C::STAGES), static_cast<uint32_t>(d / C::STAGES) & 1u,
                  DEFAULT_TIMEOUT, nullptr);
      }
      if (q_loads0 > 0) mbar_wait(bar(C::B_Q + 0), static_cast<uint32_t>(q_loads0 - 1) & 1u, DEFAULT_TIMEOUT, nullptr);
      if (q_loads1 > 0) mbar_wait(bar(C::B_Q + 1), static_cast<uint32_t>(q_loads1 - 1) & 1u, DEFAULT_TIMEOUT, nullptr);
    }
  } else if (warp == MMA_WARP || (HALVES == 1 && warp == MMA_WARP2)) {
    reg_dealloc<regs_other<D>()>();
    // -------------------------------------------------------------- MMA issuer(s)
    const bool second = (warp == MMA_WARP2);  // issues Q tile 1's MMAs with two issuers
    if (lane == 0 && (!second || issuers == 2)) {
      constexpr uint32_t idesc_qk = idesc_f16(BF16, BM, BN, false);
      constexpr uint32_t idesc_pv = idesc_f16(BF16, BM, D, true);
      // Descriptors of the tile bases; a byte offset o inside shared memory adds o >> 4 to
      // the 14-bit start-address field (addresses stay below 256 KiB, so it never carries).
      const uint64_t dq_base = sdesc_sw128(sbase + C::OFF_Q, 16, 1024);
      const uint64_t dk_base = sdesc_sw128(sbase + C::OFF_KV, 16, 1024);
      const uint64_t dv_base = sdesc_sw128(sbase + C::OFF_KV, C::CHUNK_BYTES, 1024);
      auto issue_qk = [&](int t, int st) {
        const int qt = dual ? 0 : t;  // dual: both tiles multiply Q tile 0
        const uint64_t qd = dq_base + static_cast<uint64_t>((qt * C::TILE_BYTES) >> 4);
        const uint64_t kd = dk_base + static_cast<uint64_t>((st * C::TILE_BYTES) >> 4);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t off = static_cast<uint64_t>(((kk >> 2) * C::CHUNK_BYTES + (kk & 3) * 32) >> 4);
          mma_ss(tmem + t * BN, qd + off, kd + off, idesc_qk, kk > 0 ? 1u : 0u);
        }
      };
      // k-steps [kk0, kk1) of each softmax warp's SCOLS scores: 16 scores each, P packed
      // 2 per TMEM column at t * BN + h * SCOLS + P_OFF, V rows h * SCOLS + 16 * kk.
      auto issue_pv = [&](int t, int st, bool acc, int kk0, int kk1) {
        const uint64_t vd = dv_base + static_cast<uint64_t>((st * C::TILE_BYTES) >> 4);
#pragma unroll
        for (int h = 0; h < HALVES; ++h) {
#pragma unroll
          for (int kk = kk0; kk < kk1; ++kk) {
            const int k0 = h * SCOLS + kk * 16;  // first score (V row) of this k-step
            const uint32_t p_col = C::SEP_P ? C::TMEM_P + t * (BN / 2) + kk * 8 : t * BN + h * SCOLS + P_OFF + kk * 8;
            mma_ts(tmem + C::TMEM_O + t * D, tmem + p_col, vd + static_cast<uint64_t>((k0 * 128) >> 4), idesc_pv,
                   (acc || k0 > 0) ? 1u : 0u);
          }
        }
      };
      auto mwait = [&](int b_idx, uint32_t parity) -> bool {
        return FA2_MMA_SPIN ? mbar_wait_spin(bar(b_idx), parity, a.timeout, a.err)
                            : mbar_wait(bar(b_idx), parity, a.timeout, a.err);
      };
      // PV of tile t in two parts: the k-steps reading each softmax warp's first P_SPLIT_W
      // 32-score chunks, which the warps hand over before computing the rest, then the others.
      [[maybe_unused]] int tr_n = 0, tr_j = 0;  // unit and step of the stamps (FA2_TRACE)
      auto pv_tile = [&](int t, int st, bool acc, uint32_t pph) -> bool {
        if (!mwait(C::B_P_FULL + t, pph)) return false;
        FA2_STAMP(tr_n, tr_j, t, 7);
        tc_fence_after();
        issue_pv(t, st, acc, 0, 2 * P_SPLIT_W);
        FA2_STAMP(tr_n, tr_j, t, 8);
        if (!mwait(C::B_P_LATE + t, pph)) return false;
        FA2_STAMP(tr_n, tr_j, t, 9);
        tc_fence_after();
        issue_pv(t, st, acc, 2 * P_SPLIT_W, SCOLS / 16);
        FA2_STAMP(tr_n, tr_j, t, 10);
        return true;
      };
      auto kv_wait = [&](int i) -> bool {
        return mwait(C::B_KV_FULL + i % C::STAGES, static_cast<uint32_t>(i / C::STAGES) & 1u);
      };
      Unit u;
      int slot = 0;
      next_unit<CAUSAL, VARLEN>(a, slot, u);
      if (dual) {
        // One unit. Each K/V tile feeds one Q tile; ci walks the ring in the loader's order.
        int ci = 0;
        auto take = [&]() -> int {
          const int slot = ci++;
          return kv_wait(slot) ? slot % C::STAGES : -1;
        };
        do {
          if (!mwait(C::B_Q + 0, 0)) { ok = false; break; }
          int sa = take();
          if (sa < 0) { ok = false; break; }
          tc_fence_after();
          issue_qk(0, sa);
          mma_commit(bar(C::B_S_FULL + 0));
          mma_commit(bar(C::B_KV_EMPTY + sa));
          int sb = take();
          if (sb < 0) { ok = false; break; }
          tc_fence_after();
          issue_qk(1, sb);
          mma_commit(bar(C::B_S_FULL + 1));
          mma_commit(bar(C::B_KV_EMPTY + sb));
          for (int j = 0; j < u.J; ++j) {
            const bool more = (j + 1 < u.J);
            const uint32_t pph = static_cast<uint32_t>(j) & 1u;
            for (int t = 0; t < 2; ++t) {
              const int sv = take();
              if (sv < 0 || !pv_tile(t, sv, j > 0, pph)) { ok = false; break; }
              mma_commit(bar(C::B_KV_EMPTY + sv));
              if (more) {
                const int sk = take();
                if (sk < 0) { ok = false; break; }
                tc_fence_after();
                issue_qk(t, sk);
                mma_commit(bar(C::B_S_FULL + t));
                mma_commit(bar(C::B_KV_EMPTY + sk));
              } else {
                mma_commit(bar(C::B_O_FULL + t));
              }
            }
            if (!ok) break;
          }
        } while (false);
      } else if (C::SEP_P && issuers == 1) {
        // P in its own TMEM columns: in step j the next QK of each tile (step j + 1, or the next
        // unit's step 0) goes first, as soon as that tile's softmax warps have read S_t(j)
        // (S_EMPTY); then PV(0, j) and PV(1, j) as P arrives. Each PV is followed by a commit on
        // P_EMPTY(t), which lets the softmax warps rewrite P_t and rescale O_t. Ring order stays
        // the loader's (K_j, V_j, K_j+1, ...): K_j+1 is consumed before V_j.
        do {
          if (!mwait(C::B_Q + 0, 0) || !kv_wait(0)) { ok = false; break; }
          tc_fence_after();
          issue_qk(0, 0);
          mma_commit(bar(C::B_S_FULL + 0));
          if (u.J == 1) mma_commit(bar(C::B_Q_EMPTY + 0));
          if (!mwait(C::B_Q + 1, 0)) { ok = false; break; }
          tc_fence_after();
          issue_qk(1, 0);
          mma_commit(bar(C::B_S_FULL + 1));
          mma_commit(bar(C::B_KV_EMPTY + 0));
          if (u.J == 1) mma_commit(bar(C::B_Q_EMPTY + 1));
          int n = 0, i = 0, g = 0;  // unit, ring position of its K_0, steps of the units before
          while (true) {
            Unit nx;
            int slot_next = slot;
            const bool has_next = next_unit<CAUSAL, VARLEN>(a, slot_next, nx);
            const uint32_t qph_next = static_cast<uint32_t>(n + 1) & 1u;
            for (int j = 0; j < u.J; ++j) {
              const bool last = (j + 1 == u.J);
              const int iv = i + 2 * j + 1, ik = i + 2 * j + 2;
              const int sv = iv % C::STAGES, sk = ik % C::STAGES;
              const bool more = !last || has_next;
              // The QK issued here is its unit's last one for tile t: Q_t may be reloaded after it.
              const bool qk_final = last ? (has_next && nx.J == 1) : (j + 2 == u.J);
              const uint32_t pph = static_cast<uint32_t>(g + j) & 1u;
              if (more) {
                if (!kv_wait(ik)) { ok = false; break; }
                for (int t = 0; t < 2; ++t) {
                  if (!mwait(C::B_S_EMPTY + t, pph) || (last && !mwait(C::B_Q + t, qph_next))) {
                    ok = false;
                    break;
                  }
                  tc_fence_after();
                  issue_qk(t, sk);
                  mma_commit(bar(C::B_S_FULL + t));
                  if (qk_final) mma_commit(bar(C::B_Q_EMPTY + t));
                }
                if (!ok) break;
                mma_commit(bar(C::B_KV_EMPTY + sk));
              }
              if (!kv_wait(iv)) { ok = false; break; }
              for (int t = 0; t < 2; ++t) {
                if (!pv_tile(t, sv, j > 0, pph)) { ok = false; break; }
                mma_commit(bar(C::B_P_EMPTY + t));
                if (last) mma_commit(bar(C::B_O_FULL + t));
              }
              if (!ok) break;
              mma_commit(bar(C::B_KV_EMPTY + sv));
            }
            if (!ok || !has_next) break;
            i += 2 * u.J;
            g += u.J;
            ++n;
            u = nx;
            slot = slot_next;
          }
        } while (false);
      } else if (issuers == 2) {
        // One Q tile per issuing thread. Each walks the same units and ring entries, releases
        // every K/V slot once (the slot barrier expects both) and commits its tile's barriers.
        const int t = second ? 1 : 0;
        do {
          if (!mwait(C::B_Q + t, 0) || !kv_wait(0)) { ok = false; break; }
          tc_fence_after();
          issue_qk(t, 0);
          mma_commit(bar(C::B_S_FULL + t));
          mma_commit(bar(C::B_KV_EMPTY + 0));
          if (u.J == 1) mma_commit(bar(C::B_Q_EMPTY + t));
          int n = 0, i = 0, g = 0;  // unit, ring position of its K_0, steps of the units before
          while (true) {
            Unit nx;
            int slot_next = slot;
            const bool has_next = next_unit<CAUSAL, VARLEN>(a, slot_next, nx);
            const uint32_t qph_next = static_cast<uint32_t>(n + 1) & 1u;
            for (int j = 0; j < u.J; ++j) {
              const bool last = (j + 1 == u.J);
              const int iv = i + 2 * j + 1, ik = i + 2 * j + 2;  // V_j, then K_j+1 (or the next unit's K_0)
              const int sv = iv % C::STAGES, sk = ik % C::STAGES;
              const bool more = !last || has_next;
              const bool qk_final = last ? (has_next && nx.J == 1) : (j + 2 == u.J);
              const uint32_t pph = static_cast<uint32_t>(g + j) & 1u;
              if (!kv_wait(iv) || !pv_tile(t, sv, j > 0, pph)) { ok = false; break; }
              mma_commit(bar(C::B_KV_EMPTY + sv));
              if (last) mma_commit(bar(C::B_O_FULL + t));
              if (more) {
                if ((last && !mwait(C::B_Q + t, qph_next)) || !kv_wait(ik)) { ok = false; break; }
                tc_fence_after();
                issue_qk(t, sk);
                mma_commit(bar(C::B_S_FULL + t));
                mma_commit(bar(C::B_KV_EMPTY + sk));
                if (qk_final) mma_commit(bar(C::B_Q_EMPTY + t));
              }
            }
            if (!ok || !has_next) break;
            i += 2 * u.J;
            g += u.J;
            ++n;
            u = nx;
            slot = slot_next;
          }
        } while (false);
      } else {
        do {
          // First unit: QK of both tiles on its K_0. Later units' first QKs are issued in the
          // last step of the unit before, as the next step of one continuous stream.
          if (!mwait(C::B_Q + 0, 0) || !kv_wait(0)) { ok = false; break; }
          tc_fence_after();
          issue_qk(0, 0);
          mma_commit(bar(C::B_S_FULL + 0));
          if (u.J == 1) mma_commit(bar(C::B_Q_EMPTY + 0));
          if (!mwait(C::B_Q + 1, 0)) { ok = false; break; }
          tc_fence_after();
          issue_qk(1, 0);
          mma_commit(bar(C::B_S_FULL + 1));
          mma_commit(bar(C::B_KV_EMPTY + 0));
          if (u.J == 1) mma_commit(bar(C::B_Q_EMPTY + 1));
          int n = 0, i = 0, g = 0;  // unit, ring position of its K_0, steps of the units before
          while (true) {
            Unit nx;
            int slot_next = slot;
            const bool has_next = next_unit<CAUSAL, VARLEN>(a, slot_next, nx);
            const uint32_t qph_next = static_cast<uint32_t>(n + 1) & 1u;
            for (int j = 0; j < u.J; ++j) {
              const bool last = (j + 1 == u.J);
              // V_j, then K_j+1 (at the last step: the next unit's K_0, the next ring entry).
              const int iv = i + 2 * j + 1, ik = i + 2 * j + 2;
              const int sv = iv % C::STAGES, sk = ik % C::STAGES;
              const bool more = !last || has_next;
              // The QK issued below is its unit's last one for tile t: Q_t may be reloaded after it.
              const bool qk_final = last ? (has_next && nx.J == 1) : (j + 2 == u.J);
              const uint32_t pph = static_cast<uint32_t>(g + j) & 1u;
              // DEFER: the unit's first PV overwrites O_t; the softmax warps must have read the
              // previous unit's O_t (they do so during this unit's first step).
              const bool o_wait = C::DEFER && j == 0 && n > 0;
              const uint32_t oph = static_cast<uint32_t>(n - 1) & 1u;
              tr_n = n;
              tr_j = j;
              if (!kv_wait(iv)) {
                ok = false;
                break;
              }
              FA2_STAMP(n, j, 0, 6);
              if ((o_wait && !mwait(C::B_O_EMPTY + 0, oph)) || !pv_tile(0, sv, j > 0, pph)) {
                ok = false;
                break;
              }
              if (last) mma_commit(bar(C::B_O_FULL + 0));
              if (more) {
                if ((last && !mwait(C::B_Q + 0, qph_next)) || !kv_wait(ik)) { ok = false; break; }
                FA2_STAMP(n, j, 0, 11);
                tc_fence_after();
                issue_qk(0, sk);
                mma_commit(bar(C::B_S_FULL + 0));
                FA2_STAMP(n, j, 0, 12);
                if (qk_final) mma_commit(bar(C::B_Q_EMPTY + 0));
              }
              if ((o_wait && !mwait(C::B_O_EMPTY + 1, oph)) || !pv_tile(1, sv, j > 0, pph)) { ok = false; break; }
              mma_commit(bar(C::B_KV_EMPTY + sv));
              if (last) mma_commit(bar(C::B_O_FULL + 1));
              if (more) {
                if (last && !mwait(C::B_Q + 1, qph_next)) { ok = false; break; }
                FA2_STAMP(n, j, 1, 11);
                tc_fence_after();
                issue_qk(1, sk);
                mma_commit(bar(C::B_S_FULL + 1));
                FA2_STAMP(n, j, 1, 12);
                mma_commit(bar(C::B_KV_EMPTY + sk));
                if (qk_final) mma_commit(bar(C::B_Q_EMPTY + 1));
              }
            }
            if (!ok || !has_next) break;
            i += 2 * u.J;
            g += u.J;
            ++n;
            u = nx;
            slot = slot_next;
          }
        } while (false);
      }
      // Every issued MMA must retire before TMEM is released.
      mma_commit(bar(C::B_MMA_DONE));
      mbar_wait(bar(C::B_MMA_DONE), 0, DEFAULT_TIMEOUT, nullptr);
    }
  } else if (warp < SOFTMAX_WARPS) {
    reg_alloc<regs_softmax<D>()>();
    // ------------------------------------------------------------------ softmax
    // warp = t * 4 * HALVES + h * 4 + q: Q tile t, TMEM lane quadrant q (the lanes of the
    // warp's SMSP) and, with HALVES == 2, which SCOLS scores h of each row.
    const int q = warp & 3;
    const int h = (warp >> 2) & (HALVES - 1);
    const int t = warp / (4 * HALVES);
    const int r = q * 32 + lane;      // row within the tile == TMEM lane
    const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t tS = tmem + lane_addr + t * BN + h * SCOLS;            // this warp's scores
    [[maybe_unused]] const uint32_t tS_other = tmem + lane_addr + t * BN + (h ^ 1) * SCOLS;  // the other warp's (HALVES == 2)
    const uint32_t tP = C::SEP_P ? tmem + lane_addr + C::TMEM_P + t * (BN / 2) : tS + P_OFF;
    const uint32_t tO = tmem + lane_addr + C::TMEM_O + t * D;
    const float qk_scale = a.qk_scale;
    const uint64_t sc2 = f2_pack(qk_scale, qk_scale);
    // A whole warp's wait for S or O: true in every lane when the phase completed.
    auto softmax_wait = [&](uint32_t b, uint32_t parity) -> bool {
      if constexpr (D == 128 && FA2_WARP_WAIT_D128 != 0) {
        return mbar_wait_warp(b, parity, a.timeout, a.err);
      } else {
        const bool w = mbar_wait(b, parity, a.timeout, a.err);
        return __all_sync(0xffffffffu, w);
      }
    };
    constexpr int RCOLS = D / HALVES;  // O columns this warp rescales
    constexpr bool ALL_EPI = (C::EPI_WARPS == SOFTMAX_WARPS);
    const bool epi = ALL_EPI || h == 0;             // this warp writes O columns [epi_c0, + EPI_COLS)
    const int epi_c0 = ALL_EPI ? h * C::EPI_COLS : 0;
    const uint32_t so = sbase + C::OFF_STG + (ALL_EPI ? warp : t * 4 + q) * C::STG_WARP_BYTES;  // O staging

    // HALVES == 2: the two warps of a row pair (same t and q) each publish one value per row in
    // a TMEM column and read the other's once both have arrived on the pair's barrier. One
    // exchange per K/V step (the row max) and one per unit (the row sum), so the parity is a
    // running count; the wait is bounded like every other.
    uint32_t xph = 0;
    auto exchange = [&](uint32_t col_mine, uint32_t col_other, float v, float& other) -> bool {
      tmem_st1(col_mine, __float_as_uint(v));
      tmem_wait_st();
      tc_fence_before();
      const uint32_t xb = bar(C::B_XCH + t * 4 + q);
      mbar_arrive(xb);
      const bool w = mbar_wait(xb, xph, a.timeout, a.err);
      xph ^= 1u;
      if (!__all_sync(0xffffffffu, w)) return false;
      tc_fence_after();
      other = __uint_as_float(tmem_ld1_wait(col_other));
      return true;
    };

    // FA2_SEQ_EXP: tile 0's warp of this quadrant runs the exponentials of step k after tile 1's
    // of step k - 1, tile 1's after tile 0's of step k (k counts steps over all units; both tiles
    // walk the same steps). One arrival per thread on B_SEQ[t][q] when the phase is done.
    int g = 0;  // steps of the units before
    auto seq_wait = [&](int j) -> bool {
      if constexpr (FA2_SEQ_EXP == 0) {
        return true;
      } else {
        const int k = g + j;
        if (t == 0 && k == 0) return true;
        const int other = (1 - t) * 4 + q;
        const uint32_t par = static_cast<uint32_t>(t == 0 ? k - 1 : k) & 1u;
        const bool w = mbar_wait(bar(C::B_SEQ + other), par, a.timeout, a.err);
        return __all_sync(0xffffffffu, w);
      }
    };
    auto seq_done = [&]() {
      if constexpr (FA2_SEQ_EXP != 0) mbar_arrive(bar(C::B_SEQ + t * 4 + q));
    };
    // -------------------------------------------------------------- epilogue
    // O_t / l of unit eu (the en-th unit of this CTA) to its output: wait for its last PV, read
    // O_t from TMEM, scale, convert and store. false when a bounded wait expired.
    auto epilogue = [&](const Unit& eu, int en, float el, float em) -> bool {
      (void)em;
      const int e_row0 = eu.row0 + (dual ? 0 : t * BM);
      {
        if (!softmax_wait(bar(C::B_O_FULL + t), static_cast<uint32_t>(en) & 1u)) return false;
      }
      tc_fence_after();
      constexpr int EC = C::EPI_COLS / 32;  // 32-column chunks of O this warp writes
      uint32_t o[EC][32];
      auto load_o = [&]() {
#pragma unroll
        for (int c = 0; c < EC; ++c) tmem_ld32(tO + epi_c0 + c * 32, o[c]);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < EC; ++c) reg_fence32(o[c]);
      };
      // Every warp writes O (ALL_EPI): its O columns are read before the row-sum exchange, whose
      // column at D = 128 is the first of them. Otherwise (D = 64, two warps a row) the writing
      // warp reads them after it, where it uses them.
      if constexpr (ALL_EPI) load_o();
      if constexpr (C::DEFER) {
        // O_t is in registers: the next unit's first PV may overwrite it.
        tc_fence_before();
        mbar_arrive(bar(C::B_O_EMPTY + t));
      }
      float l_row = el;
      if constexpr (HALVES == 2) {
        // The row sum is the two partial sums, the first warp's first in both warps.
        float l_other;
        if (!exchange(tmem + lane_addr + C::tmem_lx(t, h), tmem + lane_addr + C::tmem_lx(t, h ^ 1), el, l_other)) {
          return false;
        }
        l_row = (h == 0) ? el + l_other : l_other + el;
      }
      if (epi) {
        if constexpr (!ALL_EPI) load_o();
        if constexpr (SPLIT) {
          // Split-KV partial: O / l in fp32 and the row's log2-sum-exp (in qk_scale units), one
          // row per thread, for the combine kernel. Rows that saw no visible column get 0, -inf.
          const bool has = (l_row > 0.0f);
          const float inv_l = has ? 1.0f / l_row : 0.0f;
          const int split_idx = dual ? 2 * static_cast<int>(blockIdx.z) + t : static_cast<int>(blockIdx.z);
          const int64_t slot = (static_cast<int64_t>(split_idx) * gridDim.x + eu.x) * a.rows_pad + e_row0 + r;
          float4* dst = reinterpret_cast<float4*>(a.o_part + slot * D + epi_c0);
#pragma unroll
          for (int c = 0; c < EC; ++c) {
#pragma unroll
            for (int v = 0; v < 8; ++v) {
              dst[c * 8 + v] = make_float4(__uint_as_float(o[c][4 * v]) * inv_l, __uint_as_float(o[c][4 * v + 1]) * inv_l,
                                           __uint_as_float(o[c][4 * v + 2]) * inv_l, __uint_as_float(o[c][4 * v + 3]) * inv_l);
            }
          }
          if (h == 0) a.lse_part[slot] = has ? em + log2f(l_row) : -INFINITY;
        } else {
          // O / l in the input dtype, 64 columns at a time through this warp's staging slot and
          // one TMA store per chunk. Lane 0 issued every store from the slot, so it alone waits
          // for the slot to have been read before it is rewritten (the next chunk's conversion
          // overlaps the read).
          constexpr int ECH = C::EPI_COLS / 64;  // 64-column chunks
          // A row that saw no key at all (a variable-length sequence without keys, bottom-right
          // rows before the first key) has l == 0 and gets zeros.
          const float inv_l = l_row > 0.0f ? 1.0f / l_row : 0.0f;
          const uint64_t inv2 = f2_pack(inv_l, inv_l);
          const int R0 = e_row0 + q * 32;  // first row of this warp
          const int pos0 = R0 >> a.pack_shift;
          const int h0 = eu.hq0 + (R0 & (a.pack - 1));
          // The warp's O box covers 32 / min(PACK, 32) positions. In a variable-length batch a box
          // that reaches past its sequence's last position would overwrite the next sequence's
          // rows (the tensor map only clips at the end of the token axis), so such a box is
          // written row by row from registers instead.
          const bool rowwise = VARLEN && a.cu_q != nullptr && pos0 + (32 >> min(a.pack_shift, 5)) > eu.n_q;
          const int my_pos = (R0 + lane) >> a.pack_shift;
          uint16_t* my_row = static_cast<uint16_t*>(a.o) + static_cast<int64_t>(eu.q0 + my_pos) * a.on +
                             static_cast<int64_t>(eu.hq0 + ((R0 + lane) & (a.pack - 1))) * a.oh + epi_c0;
          const bool my_valid = my_pos < eu.n_q;
#pragma unroll
          for (int ch = 0; ch < ECH; ++ch) {
            const uint32_t slot = so + (FA2_STG_FULL ? ch * C::STG_SLOT_BYTES : 0);
            if (!FA2_STG_FULL || ch == 0) {
              if (lane == 0) bulk_wait_read();  // the slot's previous stores have read it
              __syncwarp();
            }
#pragma unroll
            for (int v = 0; v < 8; ++v) {
              // columns ch * 64 + 8 v .. + 8 of this warp's share, as four packed pairs
              const uint32_t* src = o[2 * ch + (v >> 2)];
              uint32_t w4[4];
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int e = (v & 3) * 8 + 2 * i;
                float x0, x1;
                f2_unpack(f2_mul(f2_pack(__uint_as_float(src[e]), __uint_as_float(src[e + 1])), inv2), x0, x1);
                w4[i] = cvt_pack2<BF16>(x0, x1);
              }
              if (rowwise) {
                if (my_valid && epi_c0 + ch * 64 + v * 8 < a.d_real) {
                  *reinterpret_cast<uint4*>(my_row + ch * 64 + v * 8) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
                }
              } else {
                st_shared_v4(slot + lane * 128 + ((static_cast<uint32_t>(v) ^ static_cast<uint32_t>(lane & 7)) << 4),
                             w4[0], w4[1], w4[2], w4[3]);
              }
            }
            if (!rowwise && (!FA2_STG_FULL || ch == ECH - 1)) {
              fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0 && pos0 < eu.n_q) {
#pragma unroll
                for (int c2 = (FA2_STG_FULL ? 0 : ch); c2 <= ch; ++c2) {
                  tma_store_4d(&tmO, so + (FA2_STG_FULL ? c2 * C::STG_SLOT_BYTES : 0), epi_c0 + c2 * 64, h0,
                               eu.q0 + pos0, eu.tb);
                }
                bulk_commit();
              }
            }
          }
        }
      }
      return true;
    };
    // DEFER: the unit whose output is still to be written (by the next unit's first step).
    Unit pend;
    int pend_n = 0;
    float pend_l = 0.0f;
    bool pending = false;

    Unit u;
    int slot = 0;
    bool have = next_unit<CAUSAL, VARLEN>(a, slot, u);
    for (int n = 0; ok && have; ++n) {
      const int J = u.J;
      const int tile_row0 = u.row0 + (dual ? 0 : t * BM);  // dual: both tiles hold Q tile 0's rows
      const int kv_base = (dual && t == 1) ? u.j0b : u.j0;  // first K/V tile of this tile's range
      const int pos = (tile_row0 + r) >> a.pack_shift;      // sequence position of this row
      const int tile_pos0 = tile_row0 >> a.pack_shift;      // position of the tile's first row

      float m_use = -INFINITY;  // reference max of this row (scaled, base 2), the same in both warps of a pair
      float l = 0.0f;           // row sum over this warp's scores
      for (int j = 0; j < J; ++j) {
        if (!softmax_wait(bar(C::B_S_FULL + t), static_cast<uint32_t>(g + j) & 1u)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          if (q == 0) FA2_STAMP(n, j, t, 0);
          FA2_STAMP(n, j, t, 16 + q);
        }
        tc_fence_after();
        const int col0 = (kv_base + j) * BN;
        const bool need_causal = CAUSAL && (col0 + BN - 1 > tile_pos0 + u.coff);
        const bool need_pad = (col0 + BN > u.n_kv);
        const bool masked = need_causal || need_pad;  // uniform over the tile's warps
        int lim = u.n_kv - 1 - col0;                  // last visible column of this tile, relative
        if (CAUSAL) lim = min(lim, pos + u.coff - col0);

        // This warp's scores of the row in one batch of loads and a single wait.
        uint32_t s[NCH][32];
        if constexpr (s_load_x<D>() == 128 && NCH == 4) {
          tmem_ld128(tS, s[0], s[1], s[2], s[3]);
        } else if constexpr (s_load_x<D>() >= 64) {
#pragma unroll
          for (int c = 0; c < NCH; c += 2) tmem_ld64(tS + c * 32, s[c], s[c + 1]);
        } else {
#pragma unroll
          for (int c = 0; c < NCH; ++c) tmem_ld32(tS + c * 32, s[c]);
        }
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < NCH; ++c) reg_fence32(s[c]);
        if (lane == 0 && q == 0) FA2_STAMP(n, j, t, 1);
        if constexpr (C::SEP_P) {
          // S_t is in registers: the MMA warp may compute the next S_t over it.
          tc_fence_before();
          mbar_arrive(bar(C::B_S_EMPTY + t));
        }
        // SEP_P: P_t and O_t are still in use by PV(t) of the step before (issued after the next
        // QK); wait for it before the first P store or O rescale of this step.
        auto p_empty_wait = [&]() -> bool {
          if constexpr (C::SEP_P) {
            if (g + j > 0) {
              if (!warp_wait_pv(bar(C::B_P_EMPTY + t), static_cast<uint32_t>(g + j - 1) & 1u, a)) return false;
              tc_fence_after();
            }
          }
          return true;
        };
        if (spec_max<D>() && !masked && j > 0 && __all_sync(0xffffffffu, m_use != -INFINITY)) {
          // P with the current reference max while the row max is taken (the two are independent
          // and use different pipes); the threshold test then runs before the hand-off.
          float m_cand = row_max_chunks(s) * qk_scale;
          if (lane == 0 && q == 0) FA2_STAMP(n, j, t, 2);
          uint64_t nm2 = f2_pack(-m_use, -m_use);
          uint64_t acc2[4];
          float alpha = 1.0f;
          // Pass 0 uses the current reference max. If some row's max moved past the threshold
          // (rare), pass 1 moves it, rescales this warp's O_t columns (PV(t, j-1) has retired:
          // S_t(j) was committed after it) and redoes these chunks with the new reference max.
          if (!seq_wait(j) || !p_empty_wait()) { ok = false; break; }
#pragma unroll 1
          for (int pass = 0;; ++pass) {
#pragma unroll
            for (int i = 0; i < 4; ++i) acc2[i] = 0;
#pragma unroll
            for (int c = 0; c < P_SPLIT_W; ++c) {
              uint32_t pk[16];
              make_p32_sum<BF16, emu_pair_mask<D, BF16>()>(s[c], sc2, nm2, pk, acc2);
              tmem_st16(tP + c * 16, pk);
            }
            if (pass == 1) break;
            if constexpr (HALVES == 2) {
              float m_other;
              if (!exchange(tS, tS_other, m_cand, m_other)) { ok = false; break; }
              m_cand = fmaxf(m_cand, m_other);
            }
            const bool bump = m_cand > m_use + RESCALE_TH;
            if (!__any_sync(0xffffffffu, bump)) break;
            if (bump) {
              alpha = ex2_mufu(m_use - m_cand);
              m_use = m_cand;
            }
            rescale_o_cols<RCOLS>(tO + h * RCOLS, alpha);
            nm2 = f2_pack(-m_use, -m_use);
          }
          if (!ok) break;
          tmem_wait_st();
          tc_fence_before();
          mbar_arrive(bar(C::B_P_FULL + t));
          if (lane == 0) { if (q == 0) FA2_STAMP(n, j, t, 3); FA2_STAMP(n, j, t, 20 + q); }
#pragma unroll
          for (int c = P_SPLIT_W; c < NCH; ++c) {
            uint32_t pk[16];
            make_p32_sum<BF16, emu_pair_mask<D, BF16>()>(s[c], sc2, nm2, pk, acc2);
            tmem_st16(tP + c * 16, pk);
          }
          tmem_wait_st();
          tc_fence_before();
          mbar_arrive(bar(C::B_P_LATE + t));
          if (lane == 0) { if (q == 0) FA2_STAMP(n, j, t, 4); FA2_STAMP(n, j, t, 24 + q); }
          seq_done();
          const uint64_t acc01 = f2_add(f2_add(acc2[0], acc2[1]), f2_add(acc2[2], acc2[3]));
          float sl0, sl1;
          f2_unpack(acc01, sl0, sl1);
          if (lane == 0 && q == 0) FA2_STAMP(n, j, t, 5);
          l = l * alpha + (sl0 + sl1);
          if (C::DEFER && pending && j == 0) {  // (not reached: the speculative path needs j > 0)
            if (!epilogue(pend, pend_n, pend_l, 0.0f)) { ok = false; break; }
            pending = false;
          }
          continue;
        }
        if (masked) {
#pragma unroll
          for (int c = 0; c < NCH; ++c) mask_chunk(s[c], h * SCOLS + c * 32, lim);
        }
        float m_cand = row_max_chunks(s) * qk_scale;
        if (lane == 0 && q == 0) FA2_STAMP(n, j, t, 2);
        if constexpr (HALVES == 2) {
          float m_other;
          if (!exchange(tS, tS_other, m_cand, m_other)) { ok = false; break; }
          m_cand = fmaxf(m_cand, m_other);
        }
        const bool bump = m_cand > m_use + RESCALE_TH;  // first tile: always (m_use = -inf)
        float alpha = 1.0f;
        if (bump) {
          alpha = ex2_mufu(m_use - m_cand);
          m_use = m_cand;
        }
        if (!p_empty_wait()) { ok = false; break; }
        if (j > 0 && __any_sync(0xffffffffu, bump)) {
          // PV(t, j-1) has retired: S_t(j) was committed after it.
          rescale_o_cols<RCOLS>(tO + h * RCOLS, alpha);
        }

        // P = exp2(s * qk_scale - m) into TMEM; the first P_SPLIT_W chunks are handed to the
        // MMA warp before the rest are computed, so PV can start on them.
        // A row that has seen only masked columns so far (possible inside a split) keeps
        // m_use = -inf; its p must be exactly 0, not exp2(-inf + inf).
        const float m_safe = (m_use == -INFINITY) ? 0.0f : m_use;
        const uint64_t nm2 = f2_pack(-m_safe, -m_safe);
        if constexpr (FA2_FFMA_PASS != 0) {
#pragma unroll
          for (int c = 0; c < NCH; ++c) {
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              float x0, x1;
              f2_unpack(f2_fma(f2_pack(__uint_as_float(s[c][2 * e]), __uint_as_float(s[c][2 * e + 1])), sc2, nm2), x0, x1);
              s[c][2 * e] = __float_as_uint(x0);
              s[c][2 * e + 1] = __float_as_uint(x1);
            }
          }
        }
        if (!seq_wait(j)) { ok = false; break; }
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
          uint32_t pk[16];
          if (masked) {
            make_p32<BF16, 0u, FA2_FFMA_PASS != 0>(s[c], sc2, nm2, pk);
          } else {
            make_p32<BF16, emu_pair_mask<D, BF16>(), FA2_FFMA_PASS != 0>(s[c], sc2, nm2, pk);
          }
          tmem_st16(tP + c * 16, pk);
          if (c == P_SPLIT_W - 1) {
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(bar(C::B_P_FULL + t));
            if (lane == 0) { if (q == 0) FA2_STAMP(n, j, t, 3); FA2_STAMP(n, j, t, 20 + q); }
          }
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(bar(C::B_P_LATE + t));
        if (lane == 0) { if (q == 0) FA2_STAMP(n, j, t, 4); FA2_STAMP(n, j, t, 24 + q); }
        seq_done();

        // Row sum of the fp32 p (before rounding, as fa2/kernel.py:98), off the critical path.
        uint64_t acc2[4] = {0, 0, 0, 0};
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            acc2[(i >> 1) & 3] =
                f2_add(acc2[(i >> 1) & 3], f2_pack(__uint_as_float(s[c][i]), __uint_as_float(s[c][i + 1])));
          }
        }
        const uint64_t acc01 = f2_add(f2_add(acc2[0], acc2[1]), f2_add(acc2[2], acc2[3]));
        float sl0, sl1;
        f2_unpack(acc01, sl0, sl1);
        if (lane == 0 && q == 0) FA2_STAMP(n, j, t, 5);
        l = l * alpha + (sl0 + sl1);
        if (C::DEFER && pending && j == 0) {
          // The previous unit's output, in the gap before this unit's S_t(1) (or the next unit).
          if (!epilogue(pend, pend_n, pend_l, 0.0f)) { ok = false; break; }
          pending = false;
        }
      }
      if (!ok) break;
      g += J;
      // The next unit, decoded while PV(t, J - 1) runs.
      Unit nu;
      have = next_unit<CAUSAL, VARLEN>(a, slot, nu);
      if constexpr (C::DEFER) {
        // This unit's output is written during the next unit's first step (or after the loop).
        pend = u;
        pend_n = n;
        pend_l = l;
        pending = true;
      } else {
        if (!epilogue(u, n, l, m_use)) { ok = false; break; }
      }
      u = nu;
    }
    if (ok && pending && !epilogue(pend, pend_n, pend_l, 0.0f)) ok = false;
    if (lane == 0) bulk_wait_all();  // the last stores have read the slot and written O
  } else {
    // The spare warps of the MMA/TMA warpgroup (warp 10 also issues with two issuers).
    reg_dealloc<regs_other<D>()>();
  }

  if (!ok && a.err != nullptr) atomicCAS(a.err, 0, FA2_ERR_TIMEOUT);  // the first report wins

  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// --------------------------------------------------------------- split-KV combine
// One warp per packed row: O = sum_s w_s O_s / sum_s w_s with w_s = 2^(lse_s - max lse), over
// the splits that cover this row's 256-row block, written in the input dtype with o's strides.
// Grid: x covers the packed rows in blocks of 8; y strides over the (batch, head block) slices
// (gridDim.y is capped at 65535 by the host, xblocks may be larger).
struct CombineArgs {
  int n_q, n_kv, pack, pack_shift, hblocks, rows_pad, num_splits, split_tiles, causal_off, xblocks;
  int bottom_right;
  int d_real;             // output columns (the caller's head dimension, <= D)
  const int* seqlens_kv;  // paged K/V: keys per sequence (n_kv and causal_off per batch); else nullptr
  int64_t ob, oh, on;     // output element strides (b, h, n); d stride is 1
};

template <int D, bool CAUSAL, bool BF16>
__global__ void __launch_bounds__(256)
fa2_combine_kernel(const float* __restrict__ o_part, const float* __restrict__ lse_part, void* out,
                   const CombineArgs c) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int R = blockIdx.x * 8 + warp;  // packed row within the (batch, head block) slice
  if (R >= c.n_q * c.pack) return;
  const int pos = R / c.pack;
  const int64_t xs = static_cast<int64_t>(c.xblocks);
  constexpr int PER = D / 32;  // columns per lane
  for (int x = static_cast<int>(blockIdx.y); x < c.xblocks; x += static_cast<int>(gridDim.y)) {
    const int b = x / c.hblocks;
    int n_kv = c.n_kv, coff = c.causal_off;
    if (c.seqlens_kv != nullptr) {
      n_kv = __ldg(c.seqlens_kv + b);
      coff = c.bottom_right ? n_kv - c.n_q : 0;
    }
    // The splits the forward kernel wrote for this row's 256-row block (at least one tile).
    const int J_cta = max(1, cta_kv_tiles<CAUSAL>(R / 256, c.n_q, n_kv, c.pack_shift, coff));
    const int ns = min(c.num_splits, (J_cta + c.split_tiles - 1) / c.split_tiles);
    const int h = (x % c.hblocks) * c.pack + R % c.pack;
    float mx = -INFINITY;
    for (int sp = 0; sp < ns; ++sp) mx = fmaxf(mx, lse_part[(sp * xs + x) * c.rows_pad + R]);
    float acc[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) acc[i] = 0.0f;
    float wsum = 0.0f;
    for (int sp = 0; sp < ns; ++sp) {
      const int64_t slot = (sp * xs + x) * c.rows_pad + R;
      const float lse = lse_part[slot];
      if (lse == -INFINITY) continue;  // this split saw no visible column of the row
      const float w = exp2f(lse - mx);
      wsum += w;
      const float* src = o_part + slot * D + lane * PER;
#pragma unroll
      for (int i = 0; i < PER; ++i) acc[i] = fmaf(w, src[i], acc[i]);
    }
    const float inv = wsum > 0.0f ? 1.0f / wsum : 0.0f;
    if (lane * PER >= c.d_real) continue;  // columns past the caller's head dimension
    uint16_t* dst = reinterpret_cast<uint16_t*>(out) + b * c.ob + h * c.oh + pos * c.on + lane * PER;
#pragma unroll
    for (int i = 0; i < PER; i += 2) {
      const uint32_t pk = cvt_pack2<BF16>(acc[i] * inv, acc[i + 1] * inv);
      *reinterpret_cast<uint32_t*>(dst + i) = pk;
    }
  }
}

}  // namespace fa2

#if FA2_PAIR != 0
#include "fa2_pair_sm100.cuh"
#endif

// =============================================================================== host

namespace {

using fa2::Cfg;

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = []() -> PFN_cuTensorMapEncodeTiled_v12000 {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult qr{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &qr) !=
            cudaSuccess ||
        qr != cudaDriverEntryPointSuccess) {
      return nullptr;
    }
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

// 4-D tiled map, 128-byte swizzle, zero fill out of bounds. dims/strides in elements.
bool make_map(CUtensorMap* m, bool bf16, const void* base, const int64_t dims[4], const int64_t strides[4],
              const uint32_t box[4]) {
  cuuint64_t gdim[4];
  cuuint64_t gstride[3];
  cuuint32_t bdim[4];
  cuuint32_t estride[4] = {1, 1, 1, 1};
  for (int i = 0; i < 4; ++i) {
    gdim[i] = static_cast<cuuint64_t>(dims[i]);
    bdim[i] = box[i];
  }
  for (int i = 1; i < 4; ++i) {
    // The stride of an extent-1 dimension is never used; give TMA a legal value.
    const int64_t s = dims[i] > 1 ? strides[i] : 8;
    gstride[i - 1] = static_cast<cuuint64_t>(s) * 2u;
  }
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  const CUresult r = fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                        const_cast<void*>(base), gdim, gstride, bdim, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

constexpr int kMaxDevices = 64;

// Streaming multiprocessors of a device (cached; 148 on B200). 0 on error.
int num_sms(int device) {
  static int cache[kMaxDevices] = {};
  if (device < 0 || device >= kMaxDevices) return 0;
  if (cache[device] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
    cache[device] = n;
  }
  return cache[device];
}

// Head dimension of the compiled kernel that serves a caller's head_dim: 16 and 32 run on the
// D = 64 build (their tensor maps are head_dim wide; TMA fills the rest of a 64-column box with
// zeros), 64 and 128 on their own.
int kernel_d(int head_dim) { return head_dim <= 64 ? 64 : 128; }

struct SplitPlan {
  int num_splits = 1, split_tiles = 0, rows_pad = 0, xblocks = 0, dual = 0, grid_z = 1;
  int64_t bytes = 0;
};

// Split layout of a call. Shapes the validation would reject (which could divide by zero
// here) get the unsplit plan, so the caller's own check reports them.
SplitPlan plan_splits(const Fa2FwdParams* p) {
  SplitPlan sp;
  if (p->num_splits <= 1) return sp;
  if (p->batch < 1 || p->heads_q < 1 || p->heads_kv < 1 || p->heads_q % p->heads_kv != 0 || p->seqlen_q < 0 ||
      p->seqlen_kv < 1) {
    return sp;
  }
  const int group = p->heads_q / p->heads_kv;
  const int pack = p->pack_gqa ? group : 1;
  const int64_t rows = static_cast<int64_t>(p->seqlen_q) * pack;
  const int mblocks = static_cast<int>((rows + 255) / 256);
  const int j_max = (p->seqlen_kv + 127) / 128;
  // Dual mode: every query row sits in the CTA's first Q tile (short queries), so the second
  // tile slot walks another split of the same rows; splits come in pairs. Under a causal mask
  // the tiles of a split past a row's last visible key are fully masked (exact zeros).
  sp.dual = (rows <= 128) ? 1 : 0;
  sp.num_splits = sp.dual ? ((p->num_splits + 1) / 2) * 2 : p->num_splits;
  sp.grid_z = sp.dual ? sp.num_splits / 2 : sp.num_splits;
  sp.split_tiles = (j_max + sp.num_splits - 1) / sp.num_splits;
  sp.rows_pad = mblocks * 256;
  sp.xblocks = p->batch * (p->heads_q / pack);
  sp.bytes = static_cast<int64_t>(sp.num_splits) * sp.xblocks * sp.rows_pad * (kernel_d(p->head_dim) + 1) * 4 + 256;
  return sp;
}

#if FA2_PAIR != 0
// CTA-pair launch (fa2_fwd_pair_kernel): clusters of two CTAs, persistent over 512-row units.
template <bool CAUSAL, bool BF16>
int launch_pair(const Fa2FwdParams* p, cudaStream_t stream, int device) {
  using PC = fa2::PairCfg;
  auto kern = fa2::fa2_fwd_pair_kernel<CAUSAL, BF16>;
  static bool attr_done[kMaxDevices] = {};
  static int max_clusters[kMaxDevices] = {};
  if (device < 0 || device >= kMaxDevices) return FA2_ERR_DEVICE;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(fa2::NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = PC::SMEM_ALLOC;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (!attr_done[device]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, PC::SMEM_ALLOC) != cudaSuccess) {
      return FA2_ERR_LAUNCH;
    }
    const int sms = num_sms(device);
    if (sms < 2) return FA2_ERR_DEVICE;
    cfg.gridDim = dim3(static_cast<unsigned>(sms & ~1), 1, 1);
    int mc = 0;
    if (cudaOccupancyMaxActiveClusters(&mc, kern, &cfg) != cudaSuccess || mc < 1) return FA2_ERR_LAUNCH;
    max_clusters[device] = mc;
    attr_done[device] = true;
  }
  const int group = p->heads_q / p->heads_kv;
  const int pack = p->pack_gqa ? group : 1;
  CUtensorMap tmQ, tmK, tmV, tmO;
  const int64_t qdims[4] = {p->head_dim, p->heads_q, p->seqlen_q, p->batch};
  const int64_t qstr[4] = {1, p->q_stride[1], p->q_stride[2], p->q_stride[0]};
  const int64_t ostr[4] = {1, p->o_stride[1], p->o_stride[2], p->o_stride[0]};
  const uint32_t gh_q = static_cast<uint32_t>(pack);
  const uint32_t qbox[4] = {64, gh_q, 128u / gh_q, 1};
  const uint32_t gh_o = static_cast<uint32_t>(pack < 32 ? pack : 32);
  const uint32_t obox[4] = {64, gh_o, 32u / gh_o, 1};
  const int64_t kdims[4] = {p->head_dim, p->seqlen_kv, p->heads_kv, p->batch};
  const int64_t kstr[4] = {1, p->k_stride[2], p->k_stride[1], p->k_stride[0]};
  const int64_t vstr[4] = {1, p->v_stride[2], p->v_stride[1], p->v_stride[0]};
  const uint32_t kbox[4] = {64, 64, 1, 1};   // half a K tile: 64 keys
  const uint32_t vbox[4] = {64, 128, 1, 1};  // half a V tile: 64 columns of d
  if (!make_map(&tmQ, BF16, p->q, qdims, qstr, qbox) || !make_map(&tmO, BF16, p->o, qdims, ostr, obox) ||
      !make_map(&tmK, BF16, p->k, kdims, kstr, kbox) || !make_map(&tmV, BF16, p->v, kdims, vstr, vbox)) {
    return FA2_ERR_TMA_ENCODE;
  }
  fa2::KArgs ka{};
  ka.n_q = p->seqlen_q;
  ka.n_kv = p->seqlen_kv;
  ka.group = group;
  ka.pack = pack;
  ka.pack_shift = 0;
  while ((1 << ka.pack_shift) < pack) ++ka.pack_shift;
  ka.hblocks = p->heads_q / pack;
  ka.bottom_right = (p->causal && p->causal_align == FA2_CAUSAL_BOTTOM_RIGHT) ? 1 : 0;
  ka.causal_off = ka.bottom_right ? p->seqlen_kv - p->seqlen_q : 0;
  ka.o = p->o;
  ka.oh = p->o_stride[1];
  ka.on = p->o_stride[2];
  ka.d_real = p->head_dim;
  ka.qk_scale = p->qk_scale;
  ka.err = p->err_flag;
  ka.gate = p->gate;
  ka.timeout = p->timeout_cycles > 0 ? p->timeout_cycles : fa2::DEFAULT_TIMEOUT;
  ka.num_splits = 1;
  const int64_t rows = static_cast<int64_t>(p->seqlen_q) * pack;
  const int64_t xblocks = static_cast<int64_t>(p->batch) * ka.hblocks;
  const int64_t mblocks = (rows + 511) / 512;
  const int64_t units = xblocks * mblocks;
  if (units > 0x7fffffffLL) return FA2_ERR_SHAPE;
  ka.xblocks = static_cast<int>(xblocks);
  ka.div_xblocks = fa2::make_fastdiv(static_cast<uint32_t>(xblocks));
  ka.div_hblocks = fa2::make_fastdiv(static_cast<uint32_t>(ka.hblocks));
  ka.div_group = fa2::make_fastdiv(static_cast<uint32_t>(group));
  ka.div_mblocks = fa2::make_fastdiv(static_cast<uint32_t>(mblocks));
  ka.mblocks = static_cast<int>(mblocks);
  ka.persistent = 1;
  ka.num_units = static_cast<int>(units);
  const int64_t clusters = units < max_clusters[device] ? units : max_clusters[device];
  cfg.gridDim = dim3(static_cast<unsigned>(2 * clusters), 1, 1);
  if (cudaLaunchKernelEx(&cfg, kern, tmQ, tmK, tmV, tmO, ka) != cudaSuccess) return FA2_ERR_LAUNCH;
  return FA2_OK;
}
#endif  // FA2_PAIR

template <int D, bool CAUSAL, bool BF16>
int launch(const Fa2FwdParams* p, cudaStream_t stream, int device) {
  const bool split = plan_splits(p).num_splits > 1;
#if FA2_PAIR != 0
  if constexpr (D == 128) {
    const int64_t pair_rows = static_cast<int64_t>(p->seqlen_q) * (p->pack_gqa ? p->heads_q / p->heads_kv : 1);
    if (!split && p->cu_seqlens_q == nullptr && p->block_table == nullptr && p->head_dim == 128 &&
        pair_rows >= FA2_PAIR_MIN_ROWS) {
      return launch_pair<CAUSAL, BF16>(p, stream, device);
    }
  }
#endif
  // Per-sequence lengths (variable-length batch or paged K/V) take the VARLEN instantiation;
  // split-KV comes with fixed lengths or paged K/V (not with cu_seqlens; validated).
  const bool per_seq = p->cu_seqlens_q != nullptr || p->block_table != nullptr;
  auto kern = split ? (per_seq ? fa2::fa2_fwd_kernel<D, CAUSAL, BF16, true, true>
                               : fa2::fa2_fwd_kernel<D, CAUSAL, BF16, true, false>)
                    : (per_seq ? fa2::fa2_fwd_kernel<D, CAUSAL, BF16, false, true>
                               : fa2::fa2_fwd_kernel<D, CAUSAL, BF16, false, false>);
  const int smem_alloc = split ? Cfg<D, true>::SMEM_ALLOC : Cfg<D, false>::SMEM_ALLOC;
  const int variant = (split ? 1 : 0) + (per_seq ? 2 : 0);
  static bool attr_done[4][kMaxDevices] = {};
  if (device < 0 || device >= kMaxDevices) return FA2_ERR_DEVICE;
  if (!attr_done[variant][device]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_alloc) != cudaSuccess) {
      return FA2_ERR_LAUNCH;
    }
    attr_done[variant][device] = true;
  }
  const int group = p->heads_q / p->heads_kv;
  const int pack = p->pack_gqa ? group : 1;

  // Q / O: dims (d, h, n, b). A box row is a (position, head) pair, heads fastest, so a
  // packed tile is exactly rows r -> (position r / PACK, head r % PACK).
  CUtensorMap tmQ, tmK, tmV, tmO;
  // Variable-length batches: one packed token axis (b extent 1) of total_q / total_kv rows.
  const bool varlen = p->cu_seqlens_q != nullptr;
  const int64_t qdims[4] = {p->head_dim, p->heads_q, varlen ? p->total_q : p->seqlen_q, varlen ? 1 : p->batch};
  const int64_t qstr[4] = {1, p->q_stride[1], p->q_stride[2], p->q_stride[0]};
  const int64_t ostr[4] = {1, p->o_stride[1], p->o_stride[2], p->o_stride[0]};
  const uint32_t gh_q = static_cast<uint32_t>(pack);           // heads per 128-row Q box
  const uint32_t qbox[4] = {64, gh_q, 128u / gh_q, 1};
  const uint32_t gh_o = static_cast<uint32_t>(pack < 32 ? pack : 32);  // 32-row O box per warp
  const uint32_t obox[4] = {64, gh_o, 32u / gh_o, 1};
  // K / V: dims (d, n, h, b), 128-row boxes of one head.
  // Paged K/V: dims (d, row in page, h, page); otherwise (d, n, h, b).
  const bool paged = p->block_table != nullptr;
  const int64_t kdims[4] = {p->head_dim, paged ? p->page_size : (varlen ? p->total_kv : p->seqlen_kv), p->heads_kv,
                            paged ? p->num_pages : (varlen ? 1 : p->batch)};
  const int64_t kstr[4] = {1, p->k_stride[2], p->k_stride[1], p->k_stride[0]};
  const int64_t vstr[4] = {1, p->v_stride[2], p->v_stride[1], p->v_stride[0]};
  const uint32_t kv_rows = static_cast<uint32_t>(paged && p->page_size < fa2::BN ? p->page_size : fa2::BN);
  const uint32_t kvbox[4] = {64, kv_rows, 1, 1};
  const bool bf16 = (p->dtype == FA2_DTYPE_BF16);
  if (!make_map(&tmQ, bf16, p->q, qdims, qstr, qbox) || !make_map(&tmO, bf16, p->o, qdims, ostr, obox) ||
      !make_map(&tmK, bf16, p->k, kdims, kstr, kvbox) || !make_map(&tmV, bf16, p->v, kdims, vstr, kvbox)) {
    return FA2_ERR_TMA_ENCODE;
  }

  fa2::KArgs ka;
  ka.n_q = p->seqlen_q;
  ka.n_kv = p->seqlen_kv;
  ka.group = group;
  ka.pack = pack;
  ka.pack_shift = 0;
  while ((1 << ka.pack_shift) < pack) ++ka.pack_shift;  // pack divides 128: a power of two
  ka.hblocks = p->heads_q / pack;
  ka.bottom_right = (p->causal && p->causal_align == FA2_CAUSAL_BOTTOM_RIGHT) ? 1 : 0;
  ka.causal_off = (ka.bottom_right && !varlen) ? p->seqlen_kv - p->seqlen_q : 0;
  ka.cu_q = p->cu_seqlens_q;
  ka.cu_kv = p->cu_seqlens_kv;
  ka.block_table = p->block_table;
  ka.seqlens_kv = p->seqlens_kv;
  ka.bt_stride = p->block_table_stride;
  ka.page_size = p->page_size;
  ka.o = p->o;
  ka.oh = p->o_stride[1];
  ka.on = p->o_stride[2];
  ka.d_real = p->head_dim;
  ka.qk_scale = p->qk_scale;
  ka.err = p->err_flag;
  ka.gate = p->gate;
  ka.timeout = p->timeout_cycles > 0 ? p->timeout_cycles : fa2::DEFAULT_TIMEOUT;
  const SplitPlan sp = plan_splits(p);
  ka.num_splits = sp.num_splits;
  ka.split_tiles = sp.split_tiles;
  ka.rows_pad = sp.rows_pad;
  ka.dual = sp.dual;
  ka.o_part = nullptr;
  ka.lse_part = nullptr;
  if (sp.num_splits > 1) {
    // workspace: [splits][x][rows_pad][D] fp32 partial O, then [splits][x][rows_pad] lse
    uint8_t* ws = static_cast<uint8_t*>(p->workspace);
    ka.o_part = reinterpret_cast<float*>(ws);
    ka.lse_part = reinterpret_cast<float*>(ws + static_cast<int64_t>(sp.num_splits) * sp.xblocks * sp.rows_pad * D * 4);
  }

  const int64_t rows = static_cast<int64_t>(p->seqlen_q) * pack;
  const int64_t xblocks = static_cast<int64_t>(p->batch) * ka.hblocks;
  const int64_t mblocks = (rows + fa2::Q_TILES * fa2::BM - 1) / (fa2::Q_TILES * fa2::BM);
  const int64_t units = xblocks * mblocks;
  ka.xblocks = static_cast<int>(xblocks);
  ka.div_xblocks = fa2::make_fastdiv(static_cast<uint32_t>(xblocks));
  ka.div_hblocks = fa2::make_fastdiv(static_cast<uint32_t>(ka.hblocks));
  ka.div_group = fa2::make_fastdiv(static_cast<uint32_t>(group));
  ka.div_mblocks = fa2::make_fastdiv(static_cast<uint32_t>(mblocks));
  ka.mblocks = static_cast<int>(mblocks);
  ka.persistent = (FA2_PERSISTENT && sp.num_splits <= 1 && units <= 0x7fffffffLL) ? 1 : 0;
  ka.num_units = ka.persistent ? static_cast<int>(units) : 0;
  dim3 grid(static_cast<unsigned>(xblocks), static_cast<unsigned>(mblocks), static_cast<unsigned>(sp.grid_z));
  if (ka.persistent) {
    const int sms = num_sms(device);
    if (sms <= 0) return FA2_ERR_DEVICE;
    grid = dim3(static_cast<unsigned>(units < sms ? units : sms), 1, 1);  // one CTA per SM
  }
  kern<<<grid, fa2::NUM_THREADS, smem_alloc, stream>>>(tmQ, tmK, tmV, tmO, ka);
  if (cudaGetLastError() != cudaSuccess) return FA2_ERR_LAUNCH;
  if (sp.num_splits > 1) {
    fa2::CombineArgs ca;
    ca.n_q = p->seqlen_q;
    ca.n_kv = p->seqlen_kv;
    ca.pack = pack;
    ca.pack_shift = ka.pack_shift;
    ca.hblocks = ka.hblocks;
    ca.rows_pad = sp.rows_pad;
    ca.num_splits = sp.num_splits;
    ca.split_tiles = sp.split_tiles;
    ca.causal_off = ka.causal_off;
    ca.bottom_right = ka.bottom_right;
    ca.d_real = p->head_dim;
    ca.seqlens_kv = paged ? p->seqlens_kv : nullptr;
    ca.xblocks = sp.xblocks;
    ca.ob = p->o_stride[0];
    ca.oh = p->o_stride[1];
    ca.on = p->o_stride[2];
    const dim3 cgrid(static_cast<unsigned>((rows + 7) / 8), static_cast<unsigned>(sp.xblocks < 65535 ? sp.xblocks : 65535));
    fa2::fa2_combine_kernel<D, CAUSAL, BF16><<<cgrid, 256, 0, stream>>>(ka.o_part, ka.lse_part, p->o, ca);
    if (cudaGetLastError() != cudaSuccess) return FA2_ERR_LAUNCH;
  }
  return FA2_OK;
}

template <int D>
int dispatch_d(const Fa2FwdParams* p, cudaStream_t s, int dev) {
  const bool bf16 = p->dtype == FA2_DTYPE_BF16;
  if (p->causal) return bf16 ? launch<D, true, true>(p, s, dev) : launch<D, true, false>(p, s, dev);
  return bf16 ? launch<D, false, true>(p, s, dev) : launch<D, false, false>(p, s, dev);
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

// Strides of a [B, H, N, D] operand: d stride 1, others multiples of 8 elements (16 B),
// non-negative. Extent-1 dimensions are exempt (their stride is never used).
bool layout_ok(const int64_t st[4], const int64_t ext[4]) {
  if (ext[3] > 1 && st[3] != 1) return false;
  for (int i = 0; i < 3; ++i) {
    if (ext[i] <= 1) continue;
    if (st[i] < 0 || (st[i] % 8) != 0 || st[i] >= (int64_t(1) << 38)) return false;
  }
  return true;
}

}  // namespace

extern "C" {

int fa2_sm100_abi_version(void) { return FA2_SM100_ABI_VERSION; }

#if FA2_TRACE
// Step-timing builds only (FA2_TRACE=1): copy out / clear the stamps of the last launch.
__attribute__((visibility("default"))) int fa2_trace_read(void* dst, int64_t bytes) {
  if (bytes > static_cast<int64_t>(sizeof(fa2::g_fa2_trace))) bytes = sizeof(fa2::g_fa2_trace);
  return cudaMemcpyFromSymbol(dst, fa2::g_fa2_trace, static_cast<size_t>(bytes)) == cudaSuccess ? 0 : 1;
}
__attribute__((visibility("default"))) int fa2_trace_clear(void) {
  static const long long zero[sizeof(fa2::g_fa2_trace) / sizeof(long long)] = {};
  return cudaMemcpyToSymbol(fa2::g_fa2_trace, zero, sizeof(fa2::g_fa2_trace)) == cudaSuccess ? 0 : 1;
}
#endif


int64_t fa2_sm100_params_size(void) { return static_cast<int64_t>(sizeof(Fa2FwdParams)); }

const char* fa2_sm100_strerror(int status) {
  switch (status) {
    case FA2_OK: return "ok";
    case FA2_ERR_NULL: return "a required pointer is NULL";
    case FA2_ERR_SHAPE: return "invalid shape (sizes, batch/head_dim mismatch, causal top-left with N_q != N_kv, or causal bottom-right with N_q > N_kv)";
    case FA2_ERR_DTYPE: return "dtype must be fp16 or bf16";
    case FA2_ERR_HEAD_DIM: return "head_dim not supported by the compiled sm_100a kernels (16, 32, 64, 128)";
    case FA2_ERR_GQA: return "H_q must be divisible by H_kv";
    case FA2_ERR_PACK: return "pack_gqa needs the GQA group to divide BLOCK_M (128)";
    case FA2_ERR_SCALE: return "qk_scale must be finite and > 0";
    case FA2_ERR_LAYOUT: return "strides/alignment not usable by TMA (d stride 1, others multiples of 16 bytes, 16-byte aligned bases)";
    case FA2_ERR_TMA_ENCODE: return "cuTensorMapEncodeTiled rejected a tensor map";
    case FA2_ERR_LAUNCH: return "kernel launch failed";
    case FA2_ERR_DEVICE: return "current device is not sm_100 (B200) or the CUDA driver entry point is missing";
    case FA2_ERR_TIMEOUT: return "a bounded wait inside the kernel expired";
    case FA2_ERR_WORKSPACE: return "num_splits > 1 needs a 16-byte aligned workspace of fa2_fwd_sm100_workspace_bytes() bytes";
    case FA2_ERR_SCRATCH_LIMIT: return "fa2_fwd_sm100_noalloc: this call needs more split-KV scratch than the library's 32 MiB static array; use fewer splits or fa2_fwd_sm100 with a workspace";
    default: return "unknown fa2_sm100 status";
  }
}

int fa2_fwd_sm100_config(int32_t head_dim, int32_t* block_m, int32_t* block_n, int32_t* threads,
                         int32_t* stages, int32_t* smem_bytes) {
  int st = 0, sm = 0;
  if (head_dim == 16 || head_dim == 32 || head_dim == 64) {
    st = Cfg<64>::STAGES;
    sm = Cfg<64>::SMEM_ALLOC;
  } else if (head_dim == 128) {
    st = Cfg<128>::STAGES;
    sm = Cfg<128>::SMEM_ALLOC;
  } else {
    return FA2_ERR_HEAD_DIM;
  }
  if (block_m) *block_m = fa2::BM;
  if (block_n) *block_n = fa2::BN;
  if (threads) *threads = fa2::NUM_THREADS;
  if (stages) *stages = st;
  if (smem_bytes) *smem_bytes = sm;
  return FA2_OK;
}

}  // extern "C"

namespace {
// Everything fa2_fwd_sm100_check validates except the split-KV workspace.
int check_core(const Fa2FwdParams* p) {
  if (p == nullptr || p->q == nullptr || p->k == nullptr || p->v == nullptr || p->o == nullptr) return FA2_ERR_NULL;
  if (p->batch < 1 || p->heads_q < 1 || p->heads_kv < 1 || p->seqlen_q < 0 || p->seqlen_kv < 1) return FA2_ERR_SHAPE;
  if (p->causal_align != FA2_CAUSAL_TOP_LEFT && p->causal_align != FA2_CAUSAL_BOTTOM_RIGHT) return FA2_ERR_SHAPE;
  const bool varlen = p->cu_seqlens_q != nullptr || p->cu_seqlens_kv != nullptr;
  const bool paged = p->block_table != nullptr || p->seqlens_kv != nullptr;
  if (varlen && paged) return FA2_ERR_SHAPE;  // paged K/V come with fixed-length queries
  if (varlen) {
    // Per-sequence lengths live on the device; the causal mask applies per sequence, with its
    // alignment, whatever the lengths. Split-KV is not offered for variable-length batches.
    if (p->cu_seqlens_q == nullptr || p->cu_seqlens_kv == nullptr) return FA2_ERR_NULL;
    if (p->total_q < 0 || p->total_kv < 1 || p->num_splits > 1) return FA2_ERR_SHAPE;
  } else if (paged) {
    // Keys per sequence on the device (at most seqlen_kv); the causal mask applies per sequence.
    if (p->block_table == nullptr || p->seqlens_kv == nullptr) return FA2_ERR_NULL;
    const int ps = p->page_size;
    if (!(ps == 16 || ps == 32 || ps == 64 || (ps >= 128 && ps % 128 == 0))) return FA2_ERR_SHAPE;
    if (p->num_pages < 1 || p->block_table_stride < (p->seqlen_kv + ps - 1) / ps) return FA2_ERR_SHAPE;
  } else {
    if (p->causal && p->causal_align == FA2_CAUSAL_TOP_LEFT && p->seqlen_q != p->seqlen_kv) return FA2_ERR_SHAPE;
    if (p->causal && p->causal_align == FA2_CAUSAL_BOTTOM_RIGHT && p->seqlen_q > p->seqlen_kv) return FA2_ERR_SHAPE;
  }
  if (p->dtype != FA2_DTYPE_FP16 && p->dtype != FA2_DTYPE_BF16) return FA2_ERR_DTYPE;
  if (p->head_dim != 16 && p->head_dim != 32 && p->head_dim != 64 && p->head_dim != 128) return FA2_ERR_HEAD_DIM;
  if (p->heads_q % p->heads_kv != 0) return FA2_ERR_GQA;
  const int group = p->heads_q / p->heads_kv;
  if (p->pack_gqa && (fa2::BM % group) != 0) return FA2_ERR_PACK;
  if (!(std::isfinite(p->qk_scale) && p->qk_scale > 0.0f)) return FA2_ERR_SCALE;
  const int pack = p->pack_gqa ? group : 1;
  const int64_t rows = static_cast<int64_t>(p->seqlen_q) * pack;
  if ((rows + 255) / 256 > 65535) return FA2_ERR_SHAPE;
  if (static_cast<int64_t>(p->batch) * (p->heads_q / pack) > 0x7fffffffLL) return FA2_ERR_SHAPE;
  const int64_t qext[4] = {varlen ? 1 : p->batch, p->heads_q, varlen ? p->total_q : p->seqlen_q, p->head_dim};
  const int64_t kext[4] = {paged ? p->num_pages : (varlen ? 1 : p->batch), p->heads_kv,
                           paged ? p->page_size : (varlen ? p->total_kv : p->seqlen_kv), p->head_dim};
  if (!layout_ok(p->q_stride, qext) || !layout_ok(p->o_stride, qext) || !layout_ok(p->k_stride, kext) ||
      !layout_ok(p->v_stride, kext)) {
    return FA2_ERR_LAYOUT;
  }
  if (!aligned16(p->q) || !aligned16(p->k) || !aligned16(p->v) || !aligned16(p->o)) return FA2_ERR_LAYOUT;
  if (p->num_splits > 256) return FA2_ERR_SHAPE;
  return FA2_OK;
}
}  // namespace

extern "C" {

int fa2_fwd_sm100_check(const Fa2FwdParams* p) {
  const int rc = check_core(p);
  if (rc != FA2_OK) return rc;
  if (p->num_splits > 1) {
    if (p->workspace == nullptr || !aligned16(p->workspace) ||
        p->workspace_bytes < plan_splits(p).bytes) {
      return FA2_ERR_WORKSPACE;
    }
  }
  return FA2_OK;
}

int64_t fa2_fwd_sm100_workspace_bytes(const Fa2FwdParams* p) {
  if (p == nullptr) return 0;
  return plan_splits(p).bytes;
}

int fa2_fwd_sm100(const Fa2FwdParams* p, void* stream) {
  const int rc = fa2_fwd_sm100_check(p);
  if (rc != FA2_OK) return rc;
  if (p->seqlen_q == 0 || (p->cu_seqlens_q != nullptr && p->total_q == 0)) return FA2_OK;
  int dev = -1, major = 0, minor = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return FA2_ERR_DEVICE;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) {
    return FA2_ERR_DEVICE;
  }
  if (major != 10 || minor != 0) return FA2_ERR_DEVICE;
  if (encode_fn() == nullptr) return FA2_ERR_DEVICE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return kernel_d(p->head_dim) == 64 ? dispatch_d<64>(p, s, dev) : dispatch_d<128>(p, s, dev);
}

}  // extern "C"

// ============================================================ allocation-free entry point
// Split-KV scratch owned by the library, for callers that cannot allocate device memory
// (see fa2_fwd_sm100_noalloc in fa2_sm100.h). In host code `g_noalloc_scratch` is only a
// host-side stand-in for the symbol, never a device address: the address comes from
// cudaGetSymbolAddress, looked up once per device below.
static __device__ __align__(256) uint8_t g_noalloc_scratch[FA2_NOALLOC_SCRATCH_BYTES];

namespace {
void* g_noalloc_addr[kMaxDevices] = {};
}  // namespace

extern "C" int fa2_fwd_sm100_noalloc(const Fa2FwdParams* p, void* stream) {
  // Shapes first: the split plan below divides by the head counts.
  const int rc = check_core(p);
  if (rc != FA2_OK) return rc;
  Fa2FwdParams q = *p;
  q.workspace = nullptr;
  q.workspace_bytes = 0;
  if (q.num_splits > 1 && plan_splits(&q).bytes > FA2_NOALLOC_SCRATCH_BYTES) return FA2_ERR_SCRATCH_LIMIT;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return FA2_ERR_DEVICE;
  if (g_noalloc_addr[dev] == nullptr) {
    // Set-up on the first call on each device, whatever its num_splits, with that device
    // current and before any launch of this call.
    void* addr = nullptr;
    if (cudaGetSymbolAddress(&addr, g_noalloc_scratch) != cudaSuccess || addr == nullptr) {
      return FA2_ERR_DEVICE;
    }
    g_noalloc_addr[dev] = addr;
  }
  if (q.num_splits > 1) {
    q.workspace = g_noalloc_addr[dev];
    q.workspace_bytes = FA2_NOALLOC_SCRATCH_BYTES;
  }
  return fa2_fwd_sm100(&q, stream);
}
