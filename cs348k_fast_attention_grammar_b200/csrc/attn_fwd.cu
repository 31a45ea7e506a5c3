// Fused attention forward for sm_100a (B200):
//     O = softmax(Q K^T * scale [+ causal mask]) V        per (batch, head)
//
// Replaces the reference's six-launch cuTile pipeline (Ss, mx, e, sm, P, O
// kernels of runs/attn_full/kernels/best_it24.py:17-99, i.e. the 8 stages of
// run_attention_search.py:49-85) with one kernel that keeps S, P and O on
// chip (tensor memory) and streams K/V once per CTA.
//
// Work unit (one CTA): one (batch, head) pair and 256 query rows, held as two
// 128-row Q tiles that alternate between the tensor cores and the softmax
// warps (while one tile's softmax runs, the tensor core works on the other
// tile's GEMMs).  Warp roles (12 warps, 384 threads):
//   warps 0-3  softmax for Q tile 0 (thread = one query row = one TMEM lane)
//   warps 4-7  softmax for Q tile 1
//   warp  8    TMA producer: Q tiles once, then K_j / V_j 128-key blocks into
//              a ring of shared-memory slots
//   warp  9    TMEM allocator + single-thread tcgen05.mma issuer
//   warps 10-11 idle (keep the register budget of the softmax warps)
// Tensor memory (512 columns x 128 lanes x 32 bit):
//   S_t at columns [128 t, 128 t + 128)  fp32 scores of tile t
//   P_t aliases the first 64 columns of S_t (128 bf16 probabilities per row)
//   O_t at columns [256 + D t, 256 + D t + D)  fp32 output accumulator
// Per KV block j the MMA warp issues, in this order,
//   O_0 += P_0(j-1) V_{j-1};  S_0 = Q_0 K_j^T;  O_1 += P_1(j-1) V_{j-1};  S_1 = Q_1 K_j^T
// so "S_t(j) complete" implies "O_t holds all blocks < j", which is when the
// softmax warps may rescale O_t in place.  P is published in two halves (keys
// 0-63, then 64-127), and O_t += P_t V starts on the first half while the
// softmax computes the second.
// This two-tile kernel serves D = 128; D = 64 runs attn_fwd_q4_kernel below
// (four Q tiles per CTA over 64-key blocks).
// Scheduling: (batch, head) pairs in groups of <= 32 MiB of K/V (L2-resident),
// causal units longest first within a group; one CTA per SM takes work units
// from a global counter once there are more units than SMs.
// Online softmax (exp2 domain, log2(e) folded into the scale): the running
// row maximum is only raised when a block's maximum exceeds it by more than
// 8 (a factor 256), which keeps O_t rescales rare; the final O / l is exact
// for any reference maximum.
#include <cuda_bf16.h>

#include <atomic>
#include <mutex>

#include "fa_internal.h"
#include "sm100_ptx.cuh"
#include "sm100_tmem_wide.cuh"

namespace fa {
namespace {

constexpr int kBM = 128;          // query rows per tile (= TMEM lanes)
constexpr int kBN = 128;          // keys per KV block
constexpr int kThreads = 384;
constexpr float kRescaleThreshold = 8.0f;

// Share of the softmax exponentials computed on the FMA pipe instead of MUFU:
// pair c of a row (of 64) is emulated when c % mod == mod - 1 (0 = none).
#ifndef FA_ATTN_EMU_MOD_D64
#define FA_ATTN_EMU_MOD_D64 4
#endif
#ifndef FA_ATTN_EMU_MOD_D128
#define FA_ATTN_EMU_MOD_D128 4
#endif
// 1 = pack probabilities to bf16 with integer ops (round half up), 0 = cvt.
#ifndef FA_ATTN_PACK_ALU
#define FA_ATTN_PACK_ALU 0
#endif
// Upper bound on the K/V bytes of one scheduling group of (batch, head) pairs.
// ncu on this pool: groups of 64 MiB re-read K/V from DRAM (cfg2 small case
// 270 MB read for 201 MB of Q/K/V, D = 64 case 2.2x), groups of <= 32 MiB do
// not (the L2 is split over the two dies, so half of it is what one working
// set can count on).
#ifndef FA_ATTN_GROUP_MIB
#define FA_ATTN_GROUP_MIB 32
#endif
// 1 = P is published in two halves (keys 0-63, 64-127) so the first half of
// O += P V starts while the softmax computes the second half.
#ifndef FA_ATTN_SPLIT_P
#define FA_ATTN_SPLIT_P 1
#endif
// 1 = softmax blocks after a row's first skip (D <= 64 kernel) or halve
// (two-tile kernel) the block maximum: the exponentials run against the
// running reference maximum, and a block whose row sum exceeds 2^64 (or is
// not finite) in any row of the warp is redone with the maximum taken and O
// rescaled.  Measured: D = 64 non-causal +5 %, causal equal; two-tile kernel
// causal -6 %, non-causal equal, so it is on for D <= 64 only.
#ifndef FA_ATTN_SPEC_MAX_D64
#define FA_ATTN_SPEC_MAX_D64 1
#endif
#ifndef FA_ATTN_SPEC_MAX_D128
#define FA_ATTN_SPEC_MAX_D128 0
#endif
// 1 = the D <= 64 kernel's speculative path reads its 64 scores with one
// TMEM load instead of two (measured 1-2 % slower than two).
#ifndef FA_ATTN_SPEC_LD2
#define FA_ATTN_SPEC_LD2 0
#endif
// Paired fp32 ops in the exponential loop: bit 0 = scale-and-subtract as one
// fma.f32x2 per two scores, bit 1 = row sums accumulated with add.f32x2.
#ifndef FA_ATTN_F2
#define FA_ATTN_F2 3
#endif
// 1 = FMA-pipe exponentials computed two at a time (exp2_fma_x2).
#ifndef FA_ATTN_EMU2
#define FA_ATTN_EMU2 1
#endif
// 1 = move registers from the producer/MMA warpgroup (FA_ATTN_REGS_MMA per
// thread) to the two softmax warpgroups (FA_ATTN_REGS_SOFTMAX) with
// setmaxnreg.  128 x 56 + 256 x 224 is the launch's 384 threads x 168
// registers exactly; any split must stay within that pool.
#ifndef FA_ATTN_SETMAXNREG
#define FA_ATTN_SETMAXNREG 1
#endif
#ifndef FA_ATTN_REGS_MMA
#define FA_ATTN_REGS_MMA 56
#endif
#ifndef FA_ATTN_REGS_SOFTMAX
#define FA_ATTN_REGS_SOFTMAX 224
#endif
static_assert(128 * FA_ATTN_REGS_MMA + 256 * FA_ATTN_REGS_SOFTMAX <= 384 * 168,
              "register split exceeds the two-tile kernel's launch pool");
// 1 = the attention kernels run persistent (one CTA per SM taking units from
// a global counter) when there are more units than SMs, so a unit's Q and
// first K/V tiles load, and its first S GEMMs run, while the previous unit
// ends.
#ifndef FA_ATTN_PERSIST
#define FA_ATTN_PERSIST 1
#endif
// 1 = the last partial wave of equal four-tile units runs as half units
// (see AttnParams::split_from).
#ifndef FA_ATTN_SPLIT_TAIL
#define FA_ATTN_SPLIT_TAIL 1
#endif
// Counter pairs for persistent launches, handed out round-robin per launch.
constexpr int kUnitCtrSlots = 1024;
__device__ unsigned int g_attn_unit_ctr[2 * kUnitCtrSlots];

// Degree-3 minimax (relative error) polynomial for 2^f on [-1/2, 1/2],
// max relative error 7.5e-5; fitted by fit_exp2_poly.py (Remez exchange).
constexpr float kExpC0 = 0.9999280571937561f;
constexpr float kExpC1 = 0.6932609677314758f;
constexpr float kExpC2 = 0.2426111251115799f;
constexpr float kExpC3 = 0.0551716685295105f;

// 2^x on the FMA/ALU pipes: x = j + f with j = round(x) (the 1.5 * 2^23
// addition leaves j in the low mantissa bits of t), 2^x = p(f) * 2^j with 2^j
// applied by adding j to the exponent field.  x is clamped to -125 so the
// result stays a normal number (2^-125 instead of 0 for masked scores).
__device__ __forceinline__ float exp2_fma(float x) {
  x = fmaxf(x, -125.f);
  const float t = __fadd_rn(x, 12582912.f);
  const float j = __fsub_rn(t, 12582912.f);
  const float f = __fsub_rn(x, j);
  const float p = fmaf(fmaf(fmaf(kExpC3, f, kExpC2), f, kExpC1), f, kExpC0);
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

// exp2_fma on two values at once: the same steps and roundings, with the
// floating-point ones paired (add.f32x2 / fma.f32x2; x - j as an exactly
// rounded fma with -1), so an emulated pair costs 12 instructions instead
// of 18.
// HI_CLAMP also clamps x to <= 126 (for callers whose x may exceed the
// exponent range, so that a huge x gives a huge result instead of a wrapped
// exponent field).
template <bool HI_CLAMP = false>
__device__ __forceinline__ void exp2_fma_x2(float x0, float x1, float& r0, float& r1) {
  if (HI_CLAMP) {
    x0 = fminf(x0, 126.f);
    x1 = fminf(x1, 126.f);
  }
  const uint64_t x = f2_pack(fmaxf(x0, -125.f), fmaxf(x1, -125.f));
  const uint64_t t = fadd2(x, f2_pack(12582912.f, 12582912.f));
  const uint64_t j = fadd2(t, f2_pack(-12582912.f, -12582912.f));
  const uint64_t f = ffma2(j, f2_pack(-1.f, -1.f), x);
  uint64_t q = ffma2(f2_pack(kExpC3, kExpC3), f, f2_pack(kExpC2, kExpC2));
  q = ffma2(q, f, f2_pack(kExpC1, kExpC1));
  q = ffma2(q, f, f2_pack(kExpC0, kExpC0));
  float p0, p1, t0, t1;
  f2_unpack(q, p0, p1);
  f2_unpack(t, t0, t1);
  r0 = __int_as_float(__float_as_int(p0) + (__float_as_int(t0) << 23));
  r1 = __int_as_float(__float_as_int(p1) + (__float_as_int(t1) << 23));
}

// Two non-negative finite fp32 -> bf16x2 (low half = lo) with integer ops:
// add half an ulp of bf16, keep the high 16 bits of each (round half up).
__device__ __forceinline__ uint32_t pack_bf16x2_alu(float lo, float hi) {
  const uint32_t a = __float_as_uint(lo) + 0x8000u;
  const uint32_t b = __float_as_uint(hi) + 0x8000u;
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, 0x7632;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

template <int D>
struct AttnCfg {
  static constexpr int kTileBytes = kBM * D * 2;          // one 128 x D bf16 tile
#ifndef FA_ATTN_STAGES_D128
#define FA_ATTN_STAGES_D128 4
#endif
  static constexpr int kStages = (D == 128) ? FA_ATTN_STAGES_D128 : 8;   // K/V ring slots
  static constexpr int kQOff = 0;
  static constexpr int kKVOff = 2 * kTileBytes;
  static constexpr int kBarOff = kKVOff + kStages * kTileBytes;
  // q_full, kv_full[kStages], kv_empty[kStages], s_full[2], p_full[2],
  // o_full[2], drain, p_half[2], q_empty, unit_full[2], unit_empty[2]
  static constexpr int kNumBars = 1 + 2 * kStages + 14;
  // tmem base, abort flag, unit ring (2 ints)
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kSmemBytes = kMiscOff + 16 + 1024;  // + alignment slack
  // TMEM column of S_t (P_t aliases its first 64 columns) and of O_t.
  __device__ static constexpr uint32_t col_s(int t) { return 128u * t; }
  __device__ static constexpr uint32_t col_o(int t) { return 256u + D * t; }
};

struct AttnParams {
  int B, H, S;
  int D;                  // head dim of the tensors (<= the kernel's D; the rest is zero padding)
  int n_units_per_head;   // ceil(S / 256)
  int group_q;            // scheduling groups hold group_q or group_q + 1 pairs;
  int group_r;            // the first group_r groups hold group_q + 1
  int nkv;                // ceil(S / 128)
  float scale_log2;       // scale * log2(e)
  void* o;               // bf16, or fp32 when OUT_F32
  int64_t o_sb, o_sh, o_ss;
  int* status;
  unsigned long long* trace;   // timeline buffer (trace builds only), else null
  // Persistent launches: units 0..total_units-1; CTA c runs
  // unit c first, then takes gridDim.x + atomicAdd(unit_ctr[0], 1) until that
  // passes total_units.  unit_ctr[1] counts finished CTAs; the last one resets
  // both words to zero for the next launch that uses this counter pair.
  // Null: one unit per CTA (grid = total_units).
  int total_units;
  unsigned int* unit_ctr;
  // 128-row Q tiles per work unit: the kernel's full width (2 or 4), or
  // fewer for small problems so that more SMs get a unit.
  int tiles_per_unit;
  // Four-tile kernel: units from split_from on are halves (tiles_per_unit / 2
  // tiles) of the units split_from, split_from + 1, ..., two per unit, so a
  // last partial wave of equal units runs on twice as many SMs.
  // split_from >= total_units: no split.
  int split_from;
};

// Optional timeline instrumentation (compiled out unless FA_ATTN_TRACE):
// clock64() stamps per CTA for the first kTraceCtas CTAs, slot layout
// [cta][iteration j][event].  Two-tile kernel: events 6t+0..6t+5 softmax tile
// t (wait start, S ready, row max done, exps start, exps done, P stored
// + arrived), 12+2t / 13+2t MMA tile t (P seen, S issued).  Four-tile kernel:
// events 4t+0..4t+3 softmax tile t (wait start, S ready, row max done, P
// stored + arrived).  Later units of a persistent CTA overwrite earlier ones.
// After those stamps, a per-unit record for the first kCtaTraceMax work units
// (256 query rows of one head): [SM id, start, first S seen by tile 0, last O
// ready, end, key blocks], the times from the global nanosecond timer so that
// units on different SMs line up.
#ifdef FA_ATTN_TRACE
constexpr int kTraceCtas = 8;
constexpr int kTraceEvents = 16;
constexpr int kTraceIters = 64;
constexpr int kCtaTraceMax = 8192;
constexpr int kCtaTraceFields = 6;
#define FA_TRACE(j, ev)                                                              \
  do {                                                                               \
    if (p.trace != nullptr && blockIdx.x < kTraceCtas && (j) < kTraceIters)          \
      p.trace[(blockIdx.x * kTraceIters + (j)) * kTraceEvents + (ev)] = clock64();   \
  } while (0)
#define FA_CTA_TRACE(unit, field, value)                                             \
  do {                                                                               \
    if (p.trace != nullptr && (unit) < kCtaTraceMax)                                 \
      p.trace[kTraceCtas * kTraceIters * kTraceEvents +                              \
              (unit) * kCtaTraceFields + (field)] = (value);                         \
  } while (0)
#else
#define FA_TRACE(j, ev) do { } while (0)
#define FA_CTA_TRACE(unit, field, value) do { } while (0)
#endif

// Bounded drain wait used only on the abort path: returns when the phase
// completes or after a short limit, ignoring the abort flag.
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity) {
  const unsigned long long t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > 50ull * 1000ull * 1000ull) return;
  }
}

// Epilogue store of accumulator columns [col, col + 32) of one output row,
// scaled by inv_l: fp32 (OUT_F32) or 16-bit pairs (fp16 when F16, else bf16),
// 16-byte stores; columns >= d (a multiple of 8) are padding and not written.
template <bool OUT_F32, bool F16>
__device__ __forceinline__ void store_o_chunk(void* o, int64_t row_off, int col, int d,
                                              const uint32_t (&r)[32], float inv_l) {
  if (OUT_F32) {
    uint4* dst = reinterpret_cast<uint4*>(static_cast<float*>(o) + row_off + col);
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (col + 4 * e < d)
        dst[e] = make_uint4(__float_as_uint(__uint_as_float(r[4 * e]) * inv_l),
                            __float_as_uint(__uint_as_float(r[4 * e + 1]) * inv_l),
                            __float_as_uint(__uint_as_float(r[4 * e + 2]) * inv_l),
                            __float_as_uint(__uint_as_float(r[4 * e + 3]) * inv_l));
  } else {
    uint32_t w[16];
#pragma unroll
    for (int e = 0; e < 16; ++e)
      w[e] = pack_16x2<F16>(__uint_as_float(r[2 * e]) * inv_l,
                            __uint_as_float(r[2 * e + 1]) * inv_l);
    uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(o) + row_off + col);
#pragma unroll
    for (int e = 0; e < 4; ++e)
      if (col + 8 * e < d) dst[e] = make_uint4(w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
  }
}

// Work unit u of the two-tile kernel: tiles_per_unit (2, or 1 for small
// problems) 128-row Q tiles of one (batch, head) pair.  Pairs are taken in consecutive groups of
// group_q + 1 (the first group_r groups) or group_q pairs, so the K/V of a
// group stay resident in L2.  Inside a group the units run
// query-position-major, and for causal attention the longest (last) query
// units of every head of the group go first, so the short units fill the
// tail.  nt[t] = key blocks of tile t (0 when the tile starts past S).
template <bool CAUSAL>
__device__ __forceinline__ void decode_unit(const AttnParams& p, int unit, int& b, int& h,
                                            int& q0, int nt[2]) {
  int heads_here, first_bh, r_in;
  const int big_units = (p.group_q + 1) * p.n_units_per_head;
  const int big_span = p.group_r * big_units;
  if (unit < big_span) {
    const int g = unit / big_units;
    r_in = unit - g * big_units;
    heads_here = p.group_q + 1;
    first_bh = g * heads_here;
  } else {
    const int x = unit - big_span;
    const int small_units = p.group_q * p.n_units_per_head;
    const int g = x / small_units;
    r_in = x - g * small_units;
    heads_here = p.group_q;
    first_bh = p.group_r * (p.group_q + 1) + g * p.group_q;
  }
  int qu = r_in / heads_here;
  const int bh = first_bh + (r_in - qu * heads_here);
  if (CAUSAL) qu = p.n_units_per_head - 1 - qu;
  b = bh / p.H;
  h = bh - b * p.H;
  q0 = qu * p.tiles_per_unit * kBM;
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int qs = q0 + t * kBM;
    if (t >= p.tiles_per_unit || qs >= p.S) nt[t] = 0;
    else if (CAUSAL) nt[t] = min(p.nkv, qs / kBN + 1);
    else nt[t] = p.nkv;
  }
}

// SPLIT (fp32 inputs at head dim <= 64, D = 128 here): every operand row is
// [hi | lo] -- the bf16 rounding of the fp32 value in the first 64 columns and
// the bf16 rounding of its remainder in the next 64 -- and the kernel forms
// S = Qh Kh^T + Qh Kl^T + Ql Kh^T and O = Ph Vh + Ph Vl + Pl Vh (the lo*lo
// terms are below fp32 rounding of the result), all accumulated in fp32, so
// the inputs keep about 16 significant bits instead of bf16's 8.  Ph / Pl are
// written to columns [0, 64) / [64, 128) of S_t; O uses 64 of its columns.
template <int D, bool CAUSAL, bool OUT_F32, bool F16, bool SPLIT = false>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ,
                    const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  using C = AttnCfg<D>;
  // The split mode keeps every exponential on MUFU (ex2.approx, relative
  // error ~2^-22): the FMA-pipe polynomial's 7.5e-5 would dominate its error.
  constexpr int kEmuMod = SPLIT ? 0 : (D == 64) ? FA_ATTN_EMU_MOD_D64 : FA_ATTN_EMU_MOD_D128;
  constexpr bool kPackAlu = FA_ATTN_PACK_ALU != 0 && !F16;
  constexpr bool kSpec = FA_ATTN_SPEC_MAX_D128 != 0 && !SPLIT;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t sQ = base + C::kQOff;
  const uint32_t sKV = base + C::kKVOff;
  const uint32_t bars = base + C::kBarOff;
  const uint32_t bar_q = bars;
  auto bar_kv_full = [&](int s) { return bars + 8u * (1 + s); };
  auto bar_kv_empty = [&](int s) { return bars + 8u * (1 + C::kStages + s); };
  auto bar_s_full = [&](int t) { return bars + 8u * (1 + 2 * C::kStages + t); };
  auto bar_p_full = [&](int t) { return bars + 8u * (3 + 2 * C::kStages + t); };
  auto bar_o_full = [&](int t) { return bars + 8u * (5 + 2 * C::kStages + t); };
  const uint32_t bar_drain = bars + 8u * (7 + 2 * C::kStages);
  // p_half[t] completes when the first 64 keys of P_t are in TMEM.
  auto bar_p_half = [&](int t) { return bars + 8u * (8 + 2 * C::kStages + t); };
  // q_empty completes when a unit's last S GEMMs are done (the Q tiles are free).
  const uint32_t bar_q_empty = bars + 8u * (10 + 2 * C::kStages);
  // Unit ring: the producer writes unit_slot[s] and arrives on unit_full[s];
  // the MMA thread and the eight softmax warps arrive on unit_empty[s] once
  // they have read it.  -1 ends the CTA's work.
  auto bar_unit_full = [&](int s) { return bars + 8u * (11 + 2 * C::kStages + s); };
  auto bar_unit_empty = [&](int s) { return bars + 8u * (13 + 2 * C::kStages + s); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + C::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + C::kMiscOff + 4);
  volatile int* unit_slot = reinterpret_cast<volatile int*>(gbase + C::kMiscOff + 8);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // ---- setup ----------------------------------------------------------------
  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(bar_kv_full(s), 1);
      mbar_init(bar_kv_empty(s), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(bar_s_full(t), 1);
      mbar_init(bar_p_full(t), kBM);
      mbar_init(bar_p_half(t), kBM);
      mbar_init(bar_o_full(t), 1);
    }
    mbar_init(bar_drain, 1);
    mbar_init(bar_q_empty, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar_unit_full(s), 1);
      mbar_init(bar_unit_empty(s), 1 + 8);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  if (warp == 8 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp >= 8) {
    // Warpgroup 2: producer, MMA issuer, two idle warps.
#if FA_ATTN_SETMAXNREG
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(FA_ATTN_REGS_MMA) : "memory");
#endif
  if (warp == 8) {
    // =================== TMA producer ===================
    if (elect_one()) {
      const uint64_t pol_q = l2_policy_evict_first();
      const uint64_t pol_kv = l2_policy_evict_last();
      // Launched as a programmatic dependent of the staging kernel, Q/K/V are
      // complete only after this wait (a no-op for ordinary launches).  Every
      // other role consumes what these loads bring, so it orders them too.
      grid_dependency_wait();
      int issued = 0;     // K/V tiles issued, over all units (ring position)
      int uc = 0;         // units published
      int unit = blockIdx.x;
      for (int take = 0;; ++take) {
        // Publish the unit (or -1) once the ring slot's previous entry is read.
        const int us = take & 1;
        if (take >= 2 &&
            !mbar_wait(bar_unit_empty(us), ((take >> 1) - 1) & 1, abort_flag, p.status))
          break;
        const bool done = unit >= p.total_units;
        unit_slot[us] = done ? -1 : unit;
        mbar_arrive(bar_unit_full(us));
        if (done) break;
        int b, h, q0, nt[2];
        decode_unit<CAUSAL>(p, unit, b, h, q0, nt);
        const int n = max(nt[0], nt[1]);
        // The Q tiles are free once the previous unit's last S GEMMs are done;
        // this unit's Q and first K/V tiles land while that unit finishes.
        if (uc > 0 && !mbar_wait(bar_q_empty, (uc - 1) & 1, abort_flag, p.status)) break;
        mbar_arrive_expect_tx(bar_q, (nt[1] > 0 ? 2 : 1) * C::kTileBytes);
#pragma unroll
        for (int t = 0; t < 2; ++t)
          if (nt[t] > 0)
#pragma unroll
            for (int dk = 0; dk < D / 64; ++dk)
              tma_load_4d(sQ + t * C::kTileBytes + dk * 16384, &tmQ, bar_q, dk * 64,
                          q0 + t * kBM, h, b, pol_q);
        ++uc;
        bool kv_ok = true;
        for (int i = 0; i < 2 * n; ++i) {
          const int s = issued % C::kStages;
          const uint32_t ph = (issued / C::kStages) & 1;
          if (!mbar_wait(bar_kv_empty(s), ph ^ 1u, abort_flag, p.status)) {
            kv_ok = false;
            break;
          }
          mbar_arrive_expect_tx(bar_kv_full(s), C::kTileBytes);
          const void* map = (i & 1) ? static_cast<const void*>(&tmV)
                                    : static_cast<const void*>(&tmK);
          const int j = i >> 1;
#pragma unroll
          for (int dk = 0; dk < D / 64; ++dk)
            tma_load_4d(sKV + s * C::kTileBytes + dk * 16384, map, bar_kv_full(s), dk * 64,
                        j * kBN, h, b, pol_kv);
          ++issued;
        }
        if (!kv_ok) break;
        if (p.unit_ctr == nullptr) {
          unit = p.total_units;
        } else {
          const unsigned int nx = gridDim.x + atomicAdd(p.unit_ctr, 1u);
          unit = nx < static_cast<unsigned int>(p.total_units) ? static_cast<int>(nx)
                                                               : p.total_units;
        }
      }
      if (*abort_flag) {
        // Let the copies already in flight land before the CTA exits.
        if (uc > 0) drain_wait(bar_q, (uc - 1) & 1);
        for (int i = max(0, issued - C::kStages); i < issued; ++i)
          drain_wait(bar_kv_full(i % C::kStages), (i / C::kStages) & 1);
      }
    }
    __syncwarp();
  } else if (warp == 9) {
    // =================== MMA issuer ===================
    if (elect_one()) {
      static_assert(!SPLIT || (D == 128 && !F16), "the split mode is bf16 hi/lo at D = 128");
      constexpr uint32_t kIdQK = idesc_f32acc(kBM, kBN, false, false, F16);
      constexpr uint32_t kIdPV = idesc_f32acc(kBM, SPLIT ? 64 : D, false, true, F16);
      bool ok = true;
      int it = 0;              // K/V tiles consumed, over all units (ring position)
      int pb[2] = {0, 0};      // key blocks of tile t in earlier units (P phases)
      for (int uc = 0; ok; ++uc) {
      const int us = uc & 1;
      if (!mbar_wait(bar_unit_full(us), (uc >> 1) & 1, abort_flag, p.status)) break;
      const int unit = unit_slot[us];
      mbar_arrive(bar_unit_empty(us));
      if (unit < 0) break;
      int b, h, q0, nt[2];
      decode_unit<CAUSAL>(p, unit, b, h, q0, nt);
      const int n = max(nt[0], nt[1]);
      if (!mbar_wait(bar_q, uc & 1, abort_flag, p.status)) break;
      tc_fence_after();
      int vslot = 0;
      for (int j = 0; ok && j <= n; ++j) {
        int kslot = 0;
        if (j < n) {
          kslot = it % C::kStages;
          if (!mbar_wait(bar_kv_full(kslot), (it / C::kStages) & 1, abort_flag, p.status)) {
            ok = false;
            break;
          }
          ++it;
          tc_fence_after();
        }
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          if (j >= 1 && j - 1 < nt[t]) {
            // O_t += P_t(j-1) V_{j-1}: A = P from TMEM (8 columns per K=16 step),
            // B = V tile, MN-major (d contiguous), 64-wide d atoms 16 KiB apart.
            const uint32_t vbase = sKV + vslot * C::kTileBytes;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
              // With split publication, keys 0-63 (K steps 0-3) go as soon as
              // the first half of P is stored, keys 64-127 after the rest.
              if (half == 0 && !FA_ATTN_SPLIT_P) continue;
              const uint32_t bar = (half == 0) ? bar_p_half(t) : bar_p_full(t);
              if (!mbar_wait(bar, (pb[t] + j - 1) & 1, abort_flag, p.status)) {
                ok = false;
                break;
              }
              tc_fence_after();
              if (half == 1) FA_TRACE(j - 1, 12 + 2 * t);
              const int kk0 = (FA_ATTN_SPLIT_P && half == 1) ? kBN / 32 : 0;
              const int kk1 = (half == 0) ? kBN / 32 : kBN / 16;
#pragma unroll
              for (int kk = kk0; kk < kk1; ++kk) {
                const uint64_t bdesc = sdesc_sw128(vbase + kk * 2048, 16384, 1024);
                const uint32_t acc = (j - 1 > 0 || kk > 0) ? 1u : 0u;
                if (SPLIT) {
                  // Ph Vh + Ph Vl + Pl Vh: Vl is the second 64-column atom of
                  // the V tile, Pl sits 64 columns after Ph.
                  const uint64_t vl = sdesc_sw128(vbase + 16384 + kk * 2048, 16384, 1024);
                  const uint32_t ph = tmem + C::col_s(t) + kk * 8;
                  mma_ts(tmem + C::col_o(t), ph, bdesc, kIdPV, acc);
                  mma_ts(tmem + C::col_o(t), ph, vl, kIdPV, 1u);
                  mma_ts(tmem + C::col_o(t), ph + 64, bdesc, kIdPV, 1u);
                } else {
                  mma_ts(tmem + C::col_o(t), tmem + C::col_s(t) + kk * 8, bdesc, kIdPV, acc);
                }
              }
            }
            if (!ok) break;
            if (j - 1 == nt[t] - 1) mma_commit(bar_o_full(t));
          }
          if (j < nt[t]) {
            // S_t = Q_t K_j^T: both K-major, 64-element swizzle atoms 16 KiB apart.
            const uint32_t qbase = sQ + t * C::kTileBytes;
            const uint32_t kbase = sKV + kslot * C::kTileBytes;
            if (SPLIT) {
              // Qh Kh^T + Qh Kl^T + Ql Kh^T over the 64 logical columns: hi
              // atoms at +0, lo atoms at +16 KiB.
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) {
                const uint64_t qh = sdesc_sw128(qbase + kk * 32, 16, 1024);
                const uint64_t kh = sdesc_sw128(kbase + kk * 32, 16, 1024);
                mma_ss(tmem + C::col_s(t), qh, kh, kIdQK, kk > 0 ? 1u : 0u);
                mma_ss(tmem + C::col_s(t), qh, sdesc_sw128(kbase + 16384 + kk * 32, 16, 1024),
                       kIdQK, 1u);
                mma_ss(tmem + C::col_s(t), sdesc_sw128(qbase + 16384 + kk * 32, 16, 1024), kh,
                       kIdQK, 1u);
              }
            } else {
#pragma unroll
              for (int kk = 0; kk < D / 16; ++kk) {
                const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
                mma_ss(tmem + C::col_s(t), sdesc_sw128(qbase + off, 16, 1024),
                       sdesc_sw128(kbase + off, 16, 1024), kIdQK, kk > 0 ? 1u : 0u);
              }
            }
            mma_commit(bar_s_full(t));
            FA_TRACE(j, 13 + 2 * t);
          }
        }
        if (!ok) break;
        if (j >= 1) mma_commit(bar_kv_empty(vslot));      // V_{j-1} consumed
        if (j < n) {
          mma_commit(bar_kv_empty(kslot));                // K_j consumed
          if (j == n - 1) mma_commit(bar_q_empty);        // the unit's last S GEMMs
          vslot = it % C::kStages;
          if (!mbar_wait(bar_kv_full(vslot), (it / C::kStages) & 1, abort_flag, p.status)) {
            ok = false;
            break;
          }
          ++it;
          tc_fence_after();
        }
      }
      pb[0] += nt[0];
      pb[1] += nt[1];
      }
      // Every issued MMA (and its commit arrivals) completes before teardown.
      mma_commit(bar_drain);
      drain_wait(bar_drain, 0);
    }
    __syncwarp();
  }
  } else {
#if FA_ATTN_SETMAXNREG
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(FA_ATTN_REGS_SOFTMAX) : "memory");
#endif
    // =================== softmax / correction / epilogue ===================
    const int t = warp >> 2;
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const uint32_t tS = tmem + lane_off + C::col_s(t);
    const uint32_t tO = tmem + lane_off + C::col_o(t);
    const float sl2 = p.scale_log2;
    bool ok = true;
    // Warp-uniform bounded wait: every lane waits, and the warp goes on only
    // if all lanes saw the phase complete, so an abort never splits a warp
    // ahead of the warp-wide votes and TMEM accesses below.
    auto wwait = [&](uint32_t bar, uint32_t parity) {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, p.status));
    };
    int sb = 0;   // key blocks of this tile in earlier units (S phases)
    int ou = 0;   // earlier units in which this tile had work (O phases)
    for (int uc = 0; ok; ++uc) {
    const int us = uc & 1;
    if (!wwait(bar_unit_full(us), (uc >> 1) & 1)) break;
    const int unit = unit_slot[us];
    __syncwarp();
    if (lane == 0) mbar_arrive(bar_unit_empty(us));
    if (unit < 0) break;
    int b, h, q0, nt[2];
    decode_unit<CAUSAL>(p, unit, b, h, q0, nt);
    if (t == 0 && lane == 0 && wq == 0) {
      FA_CTA_TRACE(unit, 1, globaltimer_ns());
      FA_CTA_TRACE(unit, 0, smid());
      FA_CTA_TRACE(unit, 5, max(nt[0], nt[1]));
    }
    const int qi = q0 + t * kBM + row;
    float m_ref = -INFINITY;   // reference row max, already scaled (log2 domain)
    float l = 0.f;             // running row sum of exp2(s * sl2 - m_ref)
    const int q_tile0 = q0 + t * kBM;
    for (int j = 0; j < nt[t]; ++j) {
      if (lane == 0 && wq == 0) FA_TRACE(j, 6 * t + 0);
      if (!wwait(bar_s_full(t), (sb + j) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (lane == 0 && wq == 0) FA_TRACE(j, 6 * t + 1);
      if (j == 0 && t == 0 && lane == 0 && wq == 0) FA_CTA_TRACE(unit, 2, globaltimer_ns());
      uint32_t sr[128];
      tmem_ld128_wait(tS, sr);      // all 128 scores of the row, one tcgen05.ld
      const int k0 = j * kBN;
      const bool need_mask = (k0 + kBN > p.S) || (CAUSAL && (k0 + kBN - 1 > q_tile0));
      if (need_mask) {
        const int lim = CAUSAL ? min(qi + 1, p.S) : p.S;   // keys [0, lim) visible
#pragma unroll
        for (int c = 0; c < kBN; ++c)
          if (k0 + c >= lim) sr[c] = __float_as_uint(-INFINITY);
      }
      float rs[4] = {0.f, 0.f, 0.f, 0.f};
      uint64_t rs2[2] = {0ull, 0ull};
      const uint64_t sl2x2 = f2_pack(sl2, sl2);
      uint32_t pk[2][32];
      uint32_t pl[2][32];    // SPLIT: bf16 remainders of the probabilities
      // Exponentials of one half of the row (keys 64 half .. 64 half + 63)
      // against the reference -neg_m: packed P into pk[half], sums into rs / rs2.
      auto exp_half = [&](int half, float neg_m) {
        const uint64_t negm2 = f2_pack(neg_m, neg_m);
#pragma unroll
        for (int cc = 0; cc < 32; ++cc) {
          const int c = half * 32 + cc;
          float x0, x1;
          if (FA_ATTN_F2 & 1) {
            // x = s * scale - m for two scores in one paired FMA
            f2_unpack(ffma2(f2_pack(__uint_as_float(sr[2 * c]), __uint_as_float(sr[2 * c + 1])),
                            sl2x2, negm2),
                      x0, x1);
          } else {
            x0 = fmaf(__uint_as_float(sr[2 * c]), sl2, neg_m);
            x1 = fmaf(__uint_as_float(sr[2 * c + 1]), sl2, neg_m);
          }
          // A fixed share of the pairs goes to the FMA pipe, the rest to MUFU.
          const bool emu = (kEmuMod > 0) && (c % (kEmuMod > 0 ? kEmuMod : 1) == kEmuMod - 1);
          float p0, p1;
          if (emu && FA_ATTN_EMU2) {
            exp2_fma_x2<kSpec>(x0, x1, p0, p1);
          } else {
            p0 = emu ? exp2_fma(x0) : ex2_approx(x0);
            p1 = emu ? exp2_fma(x1) : ex2_approx(x1);
          }
          if (FA_ATTN_F2 & 2)
            rs2[c & 1] = fadd2(rs2[c & 1], f2_pack(p0, p1));
          else
            rs[c & 3] += p0 + p1;
          pk[half][cc] = kPackAlu ? pack_bf16x2_alu(p0, p1) : pack_16x2<F16>(p0, p1);
          if (SPLIT)
            pl[half][cc] = pack_bf16x2(p0 - __uint_as_float(pk[half][cc] << 16),
                                       p1 - __uint_as_float(pk[half][cc] & 0xffff0000u));
        }
      };
      auto row_sum = [&]() {
        float a0, a1, b0, b1;
        f2_unpack(rs2[0], a0, a1);
        f2_unpack(rs2[1], b0, b1);
        return ((a0 + a1) + (b0 + b1)) + ((rs[0] + rs[1]) + (rs[2] + rs[3]));
      };
      // Speculative path (every block after the first): the first half is
      // exponentiated against the running reference maximum while only the
      // second half's maximum is taken; both are kept if every row's first
      // half sums to <= 2^64 and its second half's maximum is within 64
      // (log2 units) of the reference (2^15 and 8 for fp16 P), else the block
      // is redone the exact way below (all scores are still in registers).
      bool fast = kSpec && __all_sync(0xffffffffu, m_ref != -INFINITY);
      if (fast) {
        float h4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int c = kBN / 2; c < kBN; c += 8)
#pragma unroll
          for (int i = 0; i < 4; ++i)
            h4[i] = fmax3(h4[i], __uint_as_float(sr[c + 2 * i]), __uint_as_float(sr[c + 2 * i + 1]));
        exp_half(0, -m_ref);
        const float m_h1 = fmaxf(fmaxf(h4[0], h4[1]), fmaxf(h4[2], h4[3])) * sl2;
        fast = __all_sync(0xffffffffu, row_sum() <= (F16 ? 0x1p15f : 0x1p64f) &&
                                           m_h1 - m_ref <= (F16 ? 8.f : 64.f));
        if (!fast) {
#pragma unroll
          for (int i = 0; i < 4; ++i) rs[i] = 0.f;
          rs2[0] = rs2[1] = 0ull;
        }
      }
      if (!fast) {
        // Row max as four independent chains of 3-input maxima (short latency).
        float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int c = 0; c < kBN; c += 8)
#pragma unroll
          for (int i = 0; i < 4; ++i)
            mx4[i] = fmax3(mx4[i], __uint_as_float(sr[c + 2 * i]), __uint_as_float(sr[c + 2 * i + 1]));
        const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
        const float m_blk = mx * sl2;
        const float m_new = fmaxf(m_ref, m_blk);
        const bool need = (m_new - m_ref) > kRescaleThreshold;
        if (__any_sync(0xffffffffu, need)) {
          const float m_use = need ? m_new : m_ref;
          const float alpha = ex2_approx(m_ref - m_use);   // 1 if unchanged, 0 at start
          if (j > 0) {
#pragma unroll
            for (int c = 0; c < D / 32; ++c) {
              uint32_t o[32];
              tmem_ld32_wait(tO + c * 32, o);
#pragma unroll
              for (int e = 0; e < 32; ++e)
                o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
              tmem_st32(tO + c * 32, o);
            }
          }
          l *= alpha;
          m_ref = m_use;
        }
        if (lane == 0 && wq == 0) FA_TRACE(j, 6 * t + 2);
        exp_half(0, -m_ref);
      }
      if (lane == 0 && wq == 0) FA_TRACE(j, 6 * t + 3);
      if (FA_ATTN_SPLIT_P) {
        // keys 0-63 of P -> TMEM columns [0, 32); the MMA warp starts on them
        tmem_st32(tS, pk[0]);
        if (SPLIT) tmem_st32(tS + 64, pl[0]);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(bar_p_half(t));
      }
      exp_half(1, -m_ref);
      if (lane == 0 && wq == 0) FA_TRACE(j, 6 * t + 4);
      l += row_sum();
      if (!FA_ATTN_SPLIT_P) tmem_st32(tS, pk[0]);
      if (!FA_ATTN_SPLIT_P && SPLIT) tmem_st32(tS + 64, pl[0]);
      tmem_st32(tS + 32, pk[1]);
      if (SPLIT) tmem_st32(tS + 96, pl[1]);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar_p_full(t));
      if (lane == 0 && wq == 0) FA_TRACE(j, 6 * t + 5);
    }
    if (ok && nt[t] > 0 && wwait(bar_o_full(t), ou & 1)) {
      tc_fence_after();
      if (t == (nt[1] > 0 ? 1 : 0) && lane == 0 && wq == 0) FA_CTA_TRACE(unit, 3, globaltimer_ns());
      const float inv_l = 1.f / l;
      const int64_t orow_off = static_cast<int64_t>(b) * p.o_sb +
                               static_cast<int64_t>(h) * p.o_sh + static_cast<int64_t>(qi) * p.o_ss;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tmem_ld32_wait(tO + c * 32, o);
        if (qi < p.S && 32 * c < p.D)
          store_o_chunk<OUT_F32, F16>(p.o, orow_off, 32 * c, p.D, o, inv_l);
      }
      if (t == (nt[1] > 0 ? 1 : 0) && lane == 0 && wq == 0) FA_CTA_TRACE(unit, 4, globaltimer_ns());
    }
    if (nt[t] > 0) ++ou;
    sb += nt[t];
    }
  }

  // ---- teardown ---------------------------------------------------------------
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if (threadIdx.x == 0 && p.unit_ctr != nullptr) {
    // Every fetch of this CTA precedes the barrier above; the last CTA to
    // finish resets the counter pair for the next launch that uses it.
    __threadfence();
    if (atomicAdd(p.unit_ctr + 1, 1u) == gridDim.x - 1) {
      atomicExch(p.unit_ctr, 0u);
      atomicExch(p.unit_ctr + 1, 0u);
    }
  }
}

// Launch; with pdl, as a programmatic dependent of the previous kernel in the
// stream (it may start while that kernel runs; its producer waits for it).
template <typename Kern>
int launch_maybe_pdl(Kern kern, int grid, int threads, int smem, cudaStream_t stream, bool pdl,
                     const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                     const AttnParams& prm) {
  if (!pdl) {
    kern<<<grid, threads, smem, stream>>>(mq, mk, mv, prm);
    return cudaGetLastError() == cudaSuccess ? FA_OK : FA_ERR_LAUNCH;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, mq, mk, mv, prm) == cudaSuccess ? FA_OK : FA_ERR_LAUNCH;
}

template <int D, bool CAUSAL, bool OUT_F32, bool F16, bool SPLIT = false>
int launch_attn(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                const AttnParams& prm, int grid, cudaStream_t stream, bool pdl) {
  using C = AttnCfg<D>;
  auto kern = attn_fwd_kernel<D, CAUSAL, OUT_F32, F16, SPLIT>;
  static KernelPrep prep;
  int dev = 0;
  const int rc = prepare_kernel(prep, reinterpret_cast<const void*>(kern), C::kSmemBytes, &dev);
  if (rc != FA_OK) return rc;
  return launch_maybe_pdl(kern, grid, kThreads, C::kSmemBytes, stream, pdl, mq, mk, mv, prm);
}

// D = 64 kernel: four 128-row Q tiles per CTA (512 query rows) and 64-key
// blocks, so four independent S -> softmax -> P -> O += P V chains share the
// SM (the two-tile kernel above leaves MUFU, tensor pipe and issue slots all
// half idle at D = 64: each tile's chain latency, not a unit, bounds it).
// TMEM fits four tiles at D = 64 (4 x 64 S + 4 x 64 O columns) but not at
// D = 128.  20 warps: 0-15 softmax (tile w >> 2, lane quarter w & 3), 16 TMA
// producer, 17 TMEM allocator + MMA issuer, 18-19 idle.
// TMEM: S_t at 64 t (P_t over its first 32 columns), O_t at 256 + 64 t.
constexpr int kQ4Threads = 640;
constexpr int kQ4BN = 64;

// 1 = the four-tile kernel's ring slots hold a K block and the V block of
// the same keys (16 KiB, 8 slots): one wait and one release per key block in
// the MMA thread instead of two of each; 0 = K and V in separate 8 KiB slots.
#ifndef FA_ATTN_Q4_KVPAIR
#define FA_ATTN_Q4_KVPAIR 1
#endif
// 1 = the four-tile kernel moves registers from warpgroup 4 (producer, MMA
// issuer, two idle warps: FA_ATTN_Q4_REGS_CTRL each) to the 16 softmax warps
// (FA_ATTN_Q4_REGS_SOFTMAX each).  The launch holds 640 threads x 96
// registers (five warps per sub-partition); any split must stay within it.
#ifndef FA_ATTN_Q4_SETMAXNREG
#define FA_ATTN_Q4_SETMAXNREG 0
#endif
#ifndef FA_ATTN_Q4_REGS_CTRL
#define FA_ATTN_Q4_REGS_CTRL 40
#endif
#ifndef FA_ATTN_Q4_REGS_SOFTMAX
#define FA_ATTN_Q4_REGS_SOFTMAX 104
#endif
static_assert(128 * FA_ATTN_Q4_REGS_CTRL + 512 * FA_ATTN_Q4_REGS_SOFTMAX <= 640 * 96,
              "register split exceeds the four-tile kernel's launch pool");
struct AttnQ4Cfg {
  static constexpr int kTileBytes = kBM * 64 * 2;          // Q tile, 16 KiB
  static constexpr int kKVBytes = kQ4BN * 64 * 2;          // K or V block, 8 KiB
  static constexpr bool kPair = FA_ATTN_Q4_KVPAIR != 0;
  static constexpr int kSlotBytes = kPair ? 2 * kKVBytes : kKVBytes;
  static constexpr int kStages = kPair ? 8 : 16;
  static constexpr int kQOff = 0;
  static constexpr int kKVOff = 4 * kTileBytes;
  static constexpr int kBarOff = kKVOff + kStages * kSlotBytes;
  // q, kv_full[kStages], kv_empty[kStages], s_full[4], p_full[4], o_full[4],
  // drain, q_empty, unit_full[2], unit_empty[2]
  static constexpr int kNumBars = 1 + 2 * kStages + 12 + 1 + 5;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kSmemBytes = kMiscOff + 16 + 1024;
  __device__ static constexpr uint32_t col_s(int t) { return 64u * t; }
  __device__ static constexpr uint32_t col_o(int t) { return 256u + 64u * t; }
};

// Work unit u of the four-tile kernel: tiles_per_unit (4, or 2 or 1 for
// small problems) 128-row Q tiles of one (batch, head) pair, ordered as
// decode_unit orders the two-tile kernel's units.  nt[t] = 64-key blocks of tile t (0 past S).
template <bool CAUSAL>
__device__ __forceinline__ void decode_unit_q4(const AttnParams& p, int unit, int& b, int& h,
                                               int& q0, int nt[4]) {
  int half = -1;
  if (unit >= p.split_from) {
    const int x = unit - p.split_from;
    unit = p.split_from + (x >> 1);
    half = x & 1;
  }
  int heads_here, first_bh, r_in;
  const int big_units = (p.group_q + 1) * p.n_units_per_head;
  const int big_span = p.group_r * big_units;
  if (unit < big_span) {
    const int g = unit / big_units;
    r_in = unit - g * big_units;
    heads_here = p.group_q + 1;
    first_bh = g * heads_here;
  } else {
    const int x = unit - big_span;
    const int small_units = p.group_q * p.n_units_per_head;
    const int g = x / small_units;
    r_in = x - g * small_units;
    heads_here = p.group_q;
    first_bh = p.group_r * (p.group_q + 1) + g * p.group_q;
  }
  int qu = r_in / heads_here;
  const int bh = first_bh + (r_in - qu * heads_here);
  if (CAUSAL) qu = p.n_units_per_head - 1 - qu;
  b = bh / p.H;
  h = bh - b * p.H;
  q0 = qu * p.tiles_per_unit * kBM;
  int tpu = p.tiles_per_unit;
  if (half >= 0) {
    tpu >>= 1;
    q0 += half * tpu * kBM;
  }
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const int qs = q0 + t * kBM;
    if (t >= tpu || qs >= p.S) nt[t] = 0;
    else if (CAUSAL) nt[t] = min(p.nkv, (qs + kBM - 1) / kQ4BN + 1);
    else nt[t] = p.nkv;
  }
}

template <bool CAUSAL, bool OUT_F32, bool F16>
__global__ void __launch_bounds__(kQ4Threads, 1)
    attn_fwd_q4_kernel(const __grid_constant__ CUtensorMap tmQ,
                       const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  using C = AttnQ4Cfg;
  constexpr int D = 64;
  constexpr int kNT = 4;
  constexpr int kEmuMod = FA_ATTN_EMU_MOD_D64;
  constexpr bool kSpec = FA_ATTN_SPEC_MAX_D64 != 0;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t sQ = base + C::kQOff;
  const uint32_t sKV = base + C::kKVOff;
  const uint32_t bars = base + C::kBarOff;
  const uint32_t bar_q = bars;
  auto bar_kv_full = [&](int s) { return bars + 8u * (1 + s); };
  auto bar_kv_empty = [&](int s) { return bars + 8u * (1 + C::kStages + s); };
  constexpr int kB0 = 1 + 2 * C::kStages;
  auto bar_s_full = [&](int t) { return bars + 8u * (kB0 + t); };
  auto bar_p_full = [&](int t) { return bars + 8u * (kB0 + 4 + t); };
  auto bar_o_full = [&](int t) { return bars + 8u * (kB0 + 8 + t); };
  const uint32_t bar_drain = bars + 8u * (kB0 + 12);
  // q_empty: a unit's last S GEMMs are done; unit ring as in attn_fwd_kernel,
  // read by the MMA thread and the 16 softmax warps.
  const uint32_t bar_q_empty = bars + 8u * (kB0 + 13);
  auto bar_unit_full = [&](int s) { return bars + 8u * (kB0 + 14 + s); };
  auto bar_unit_empty = [&](int s) { return bars + 8u * (kB0 + 16 + s); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + C::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + C::kMiscOff + 4);
  volatile int* unit_slot = reinterpret_cast<volatile int*>(gbase + C::kMiscOff + 8);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(bar_kv_full(s), 1);
      mbar_init(bar_kv_empty(s), 1);
    }
    for (int t = 0; t < kNT; ++t) {
      mbar_init(bar_s_full(t), 1);
      mbar_init(bar_p_full(t), kBM);
      mbar_init(bar_o_full(t), 1);
    }
    mbar_init(bar_drain, 1);
    mbar_init(bar_q_empty, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar_unit_full(s), 1);
      mbar_init(bar_unit_empty(s), 1 + 16);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 17) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  if (warp == 16 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp >= 16) {
    // Warpgroup 4: producer, MMA issuer, two idle warps.
#if FA_ATTN_Q4_SETMAXNREG
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(FA_ATTN_Q4_REGS_CTRL) : "memory");
#endif
  if (warp == 16) {
    // =================== TMA producer ===================
    if (elect_one()) {
      const uint64_t pol_q = l2_policy_evict_first();
      const uint64_t pol_kv = l2_policy_evict_last();
      grid_dependency_wait();   // see attn_fwd_kernel
      int issued = 0;     // K/V blocks issued, over all units (ring position)
      int uc = 0;         // units published
      int unit = blockIdx.x;
      for (int take = 0;; ++take) {
        const int us = take & 1;
        if (take >= 2 &&
            !mbar_wait(bar_unit_empty(us), ((take >> 1) - 1) & 1, abort_flag, p.status))
          break;
        const bool done = unit >= p.total_units;
        unit_slot[us] = done ? -1 : unit;
        mbar_arrive(bar_unit_full(us));
        if (done) break;
        int b, h, q0, nt[kNT];
        decode_unit_q4<CAUSAL>(p, unit, b, h, q0, nt);
        int n = 0, ntiles = 0;
#pragma unroll
        for (int t = 0; t < kNT; ++t) {
          n = max(n, nt[t]);
          ntiles += (nt[t] > 0) ? 1 : 0;
        }
        if (uc > 0 && !mbar_wait(bar_q_empty, (uc - 1) & 1, abort_flag, p.status)) break;
        mbar_arrive_expect_tx(bar_q, ntiles * C::kTileBytes);
#pragma unroll
        for (int t = 0; t < kNT; ++t)
          if (nt[t] > 0)
            tma_load_4d(sQ + t * C::kTileBytes, &tmQ, bar_q, 0, q0 + t * kBM, h, b, pol_q);
        ++uc;
        bool kv_ok = true;
        for (int i = 0; i < (C::kPair ? n : 2 * n); ++i) {
          const int s = issued % C::kStages;
          const uint32_t ph = (issued / C::kStages) & 1;
          if (!mbar_wait(bar_kv_empty(s), ph ^ 1u, abort_flag, p.status)) {
            kv_ok = false;
            break;
          }
          mbar_arrive_expect_tx(bar_kv_full(s), C::kSlotBytes);
          if (C::kPair) {
            // K_i at the slot's start, V_i 8 KiB after it
            tma_load_4d(sKV + s * C::kSlotBytes, &tmK, bar_kv_full(s), 0, i * kQ4BN, h, b, pol_kv);
            tma_load_4d(sKV + s * C::kSlotBytes + C::kKVBytes, &tmV, bar_kv_full(s), 0,
                        i * kQ4BN, h, b, pol_kv);
          } else {
            const void* map = (i & 1) ? static_cast<const void*>(&tmV)
                                      : static_cast<const void*>(&tmK);
            tma_load_4d(sKV + s * C::kSlotBytes, map, bar_kv_full(s), 0, (i >> 1) * kQ4BN, h, b,
                        pol_kv);
          }
          ++issued;
        }
        if (!kv_ok) break;
        if (p.unit_ctr == nullptr) {
          unit = p.total_units;
        } else {
          const unsigned int nx = gridDim.x + atomicAdd(p.unit_ctr, 1u);
          unit = nx < static_cast<unsigned int>(p.total_units) ? static_cast<int>(nx)
                                                               : p.total_units;
        }
      }
      if (*abort_flag) {
        if (uc > 0) drain_wait(bar_q, (uc - 1) & 1);
        for (int i = max(0, issued - C::kStages); i < issued; ++i)
          drain_wait(bar_kv_full(i % C::kStages), (i / C::kStages) & 1);
      }
    }
    __syncwarp();
  } else if (warp == 17) {
    // =================== MMA issuer ===================
    // Per block j, for t = 0..3: O_t += P_t(j-1) V_{j-1}, then S_t = Q_t K_j^T.
    if (elect_one()) {
      constexpr uint32_t kIdQK = idesc_f32acc(kBM, kQ4BN, false, false, F16);
      constexpr uint32_t kIdPV = idesc_f32acc(kBM, D, false, true, F16);
      bool ok = true;
      int it = 0;                     // K/V blocks consumed, over all units
      int pb[kNT] = {0, 0, 0, 0};     // blocks of tile t in earlier units (P phases)
      for (int uc = 0; ok; ++uc) {
      const int us = uc & 1;
      if (!mbar_wait(bar_unit_full(us), (uc >> 1) & 1, abort_flag, p.status)) break;
      const int unit = unit_slot[us];
      mbar_arrive(bar_unit_empty(us));
      if (unit < 0) break;
      int b, h, q0, nt[kNT];
      decode_unit_q4<CAUSAL>(p, unit, b, h, q0, nt);
      int n = 0;
#pragma unroll
      for (int t = 0; t < kNT; ++t) n = max(n, nt[t]);
      if (!mbar_wait(bar_q, uc & 1, abort_flag, p.status)) break;
      tc_fence_after();
      int vslot = 0;
      for (int j = 0; ok && j <= n; ++j) {
        int kslot = 0;
        if (j < n) {
          kslot = it % C::kStages;
          if (!mbar_wait(bar_kv_full(kslot), (it / C::kStages) & 1, abort_flag, p.status)) {
            ok = false;
            break;
          }
          ++it;
          tc_fence_after();
        }
#pragma unroll
        for (int t = 0; t < kNT; ++t) {
          if (j >= 1 && j - 1 < nt[t]) {
            if (!mbar_wait(bar_p_full(t), (pb[t] + j - 1) & 1, abort_flag, p.status)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t vbase = sKV + vslot * C::kSlotBytes + (C::kPair ? C::kKVBytes : 0);
#pragma unroll
            for (int kk = 0; kk < kQ4BN / 16; ++kk) {
              const uint64_t bdesc = sdesc_sw128(vbase + kk * 2048, kQ4BN * 128, 1024);
              mma_ts(tmem + C::col_o(t), tmem + C::col_s(t) + kk * 8, bdesc, kIdPV,
                     (j - 1 > 0 || kk > 0) ? 1u : 0u);
            }
            if (j - 1 == nt[t] - 1) mma_commit(bar_o_full(t));
          }
          if (j < nt[t]) {
            const uint32_t qbase = sQ + t * C::kTileBytes;
            const uint32_t kbase = sKV + kslot * C::kSlotBytes;
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk)
              mma_ss(tmem + C::col_s(t), sdesc_sw128(qbase + kk * 32, 16, 1024),
                     sdesc_sw128(kbase + kk * 32, 16, 1024), kIdQK, kk > 0 ? 1u : 0u);
            mma_commit(bar_s_full(t));
          }
        }
        if (!ok) break;
        if (C::kPair) {
          // The slot of block j - 1 (K used by S(j - 1), V by the P V just
          // issued) is free once these MMAs complete; block j's slot serves
          // the next iteration's P V.
          if (j >= 1) mma_commit(bar_kv_empty(vslot));
          if (j == n - 1) mma_commit(bar_q_empty);        // the unit's last S GEMMs
          vslot = kslot;
          continue;
        }
        if (j >= 1) mma_commit(bar_kv_empty(vslot));
        if (j < n) {
          mma_commit(bar_kv_empty(kslot));
          if (j == n - 1) mma_commit(bar_q_empty);        // the unit's last S GEMMs
          vslot = it % C::kStages;
          if (!mbar_wait(bar_kv_full(vslot), (it / C::kStages) & 1, abort_flag, p.status)) {
            ok = false;
            break;
          }
          ++it;
          tc_fence_after();
        }
      }
#pragma unroll
      for (int t = 0; t < kNT; ++t) pb[t] += nt[t];
      }
      mma_commit(bar_drain);
      drain_wait(bar_drain, 0);
    }
    __syncwarp();
  }
  } else {
#if FA_ATTN_Q4_SETMAXNREG
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(FA_ATTN_Q4_REGS_SOFTMAX) : "memory");
#endif
    // =================== softmax / epilogue (one tile) ===================
    const int t = warp >> 2;
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const uint32_t tS = tmem + lane_off + C::col_s(t);
    const uint32_t tO = tmem + lane_off + C::col_o(t);
    const float sl2 = p.scale_log2;
    bool ok = true;
    auto wwait = [&](uint32_t bar, uint32_t parity) {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, p.status));
    };
    int sb = 0;   // blocks of this tile in earlier units (S phases)
    int ou = 0;   // earlier units in which this tile had work (O phases)
    for (int uc = 0; ok; ++uc) {
    const int us = uc & 1;
    if (!wwait(bar_unit_full(us), (uc >> 1) & 1)) break;
    const int unit = unit_slot[us];
    __syncwarp();
    if (lane == 0) mbar_arrive(bar_unit_empty(us));
    if (unit < 0) break;
    int b, h, q0, nt[kNT];
    decode_unit_q4<CAUSAL>(p, unit, b, h, q0, nt);
    const int qi = q0 + t * kBM + row;
    const int q_tile0 = q0 + t * kBM;
    float m_ref = -INFINITY;
    float l = 0.f;
    const int my_nt = nt[t];
    for (int j = 0; j < my_nt; ++j) {
      if (lane == 0 && wq == 0) FA_TRACE(j, 4 * t + 0);
      if (!wwait(bar_s_full(t), (sb + j) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (lane == 0 && wq == 0) FA_TRACE(j, 4 * t + 1);
      const int k0 = j * kQ4BN;
      const bool need_mask = (k0 + kQ4BN > p.S) || (CAUSAL && (k0 + kQ4BN - 1 > q_tile0));
      const int lim = CAUSAL ? min(qi + 1, p.S) : p.S;
      const uint64_t sl2x2 = f2_pack(sl2, sl2);
      // Exponentials of one 32-column chunk of S against reference neg_m:
      // packed probabilities into pk, row sums into rs2.
      // exp_vals: the same for 32 scores already in registers.
      auto exp_vals = [&](uint32_t* r, int ch, float neg_m, uint32_t (&pk)[16],
                          uint64_t (&rs2)[2]) {
        if (need_mask) {
#pragma unroll
          for (int c = 0; c < 32; ++c)
            if (k0 + 32 * ch + c >= lim) r[c] = __float_as_uint(-INFINITY);
        }
        const uint64_t negm2 = f2_pack(neg_m, neg_m);
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          float x0, x1;
          f2_unpack(ffma2(f2_pack(__uint_as_float(r[2 * c]), __uint_as_float(r[2 * c + 1])),
                          sl2x2, negm2),
                    x0, x1);
          const int pair = 16 * ch + c;
          const bool emu = (kEmuMod > 0) && (pair % (kEmuMod > 0 ? kEmuMod : 1) == kEmuMod - 1);
          float p0, p1;
          if (emu) {
            exp2_fma_x2<kSpec>(x0, x1, p0, p1);
          } else {
            p0 = ex2_approx(x0);
            p1 = ex2_approx(x1);
          }
          rs2[c & 1] = fadd2(rs2[c & 1], f2_pack(p0, p1));
          pk[c] = pack_16x2<F16>(p0, p1);
        }
      };
      auto exp_chunk = [&](int ch, float neg_m, uint32_t (&pk)[16], uint64_t (&rs2)[2]) {
        uint32_t r[32];
        tmem_ld32_wait(tS + 32 * ch, r);
        exp_vals(r, ch, neg_m, pk, rs2);
      };
      auto sum2 = [](const uint64_t (&rs2)[2]) {
        float a0, a1, b0, b1;
        f2_unpack(rs2[0], a0, a1);
        f2_unpack(rs2[1], b0, b1);
        return (a0 + a1) + (b0 + b1);
      };
      float l_blk = 0.f;
      // Speculative path (every block after a row's first): exponentiate
      // against the running reference maximum without taking the block
      // maximum; keep the result only if every row's block sum stays <= 2^64
      // (finite, far from fp32 overflow; 2^15 for fp16 P), else take the
      // exact path below.
      bool fast = kSpec && __all_sync(0xffffffffu, m_ref != -INFINITY);
      if (fast) {
        uint32_t pk0[16], pk1[16];
        uint64_t rs2[2] = {0ull, 0ull};
        if (FA_ATTN_SPEC_LD2) {
          uint32_t r[64];
          tmem_ld64_wait(tS, r);
          exp_vals(r, 0, -m_ref, pk0, rs2);
          exp_vals(r + 32, 1, -m_ref, pk1, rs2);
        } else {
          exp_chunk(0, -m_ref, pk0, rs2);
          exp_chunk(1, -m_ref, pk1, rs2);
        }
        l_blk = sum2(rs2);
        // (fp16 P: every probability must stay below fp16's 65504)
        fast = __all_sync(0xffffffffu, l_blk <= (F16 ? 0x1p15f : 0x1p64f));
        if (fast) {
          tmem_st16(tS, pk0);
          tmem_st16(tS + 16, pk1);
        }
      }
      if (!fast) {
        float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int ch = 0; ch < 2; ++ch) {
          uint32_t r[32];
          tmem_ld32_wait(tS + 32 * ch, r);
          if (need_mask) {
#pragma unroll
            for (int c = 0; c < 32; ++c)
              if (k0 + 32 * ch + c >= lim) r[c] = __float_as_uint(-INFINITY);
          }
#pragma unroll
          for (int c = 0; c < 32; c += 8)
#pragma unroll
            for (int i = 0; i < 4; ++i)
              mx4[i] = fmax3(mx4[i], __uint_as_float(r[c + 2 * i]), __uint_as_float(r[c + 2 * i + 1]));
        }
        const float m_blk = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * sl2;
        const bool need = (m_ref == -INFINITY) ? (m_blk > -INFINITY)
                                               : (m_blk - m_ref > kRescaleThreshold);
        if (__any_sync(0xffffffffu, need)) {
          const float m_use = need ? m_blk : m_ref;
          const float alpha = (m_ref == -INFINITY) ? 0.f : ex2_approx(m_ref - m_use);
          if (j > 0) {
#pragma unroll
            for (int c = 0; c < 2; ++c) {
              uint32_t o[32];
              tmem_ld32_wait(tO + c * 32, o);
#pragma unroll
              for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
              tmem_st32(tO + c * 32, o);
            }
            tmem_wait_st();
          }
          l *= alpha;
          m_ref = m_use;
        }
        if (lane == 0 && wq == 0) FA_TRACE(j, 4 * t + 2);
        const float neg_m = (m_ref == -INFINITY) ? 0.f : -m_ref;
        uint64_t rs2[2] = {0ull, 0ull};
#pragma unroll
        for (int ch = 0; ch < 2; ++ch) {
          uint32_t pk[16];
          exp_chunk(ch, neg_m, pk, rs2);
          tmem_st16(tS + 16 * ch, pk);
        }
        l_blk = sum2(rs2);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar_p_full(t));
      if (lane == 0 && wq == 0) FA_TRACE(j, 4 * t + 3);
      l += l_blk;
    }
    if (ok && my_nt > 0 && wwait(bar_o_full(t), ou & 1)) {
      tc_fence_after();
      const float inv_l = 1.f / l;
      const int64_t orow_off = static_cast<int64_t>(b) * p.o_sb +
                               static_cast<int64_t>(h) * p.o_sh + static_cast<int64_t>(qi) * p.o_ss;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t o[32];
        tmem_ld32_wait(tO + c * 32, o);
        if (qi < p.S && 32 * c < p.D)
          store_o_chunk<OUT_F32, F16>(p.o, orow_off, 32 * c, p.D, o, inv_l);
      }
    }
    if (my_nt > 0) ++ou;
    sb += my_nt;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 17) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if (threadIdx.x == 0 && p.unit_ctr != nullptr) {
    __threadfence();
    if (atomicAdd(p.unit_ctr + 1, 1u) == gridDim.x - 1) {
      atomicExch(p.unit_ctr, 0u);
      atomicExch(p.unit_ctr + 1, 0u);
    }
  }
}

template <bool CAUSAL, bool OUT_F32, bool F16>
int launch_attn_q4(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                   const AttnParams& prm, int grid, cudaStream_t stream, bool pdl) {
  using C = AttnQ4Cfg;
  auto kern = attn_fwd_q4_kernel<CAUSAL, OUT_F32, F16>;
  static KernelPrep prep;
  int dev = 0;
  const int rc = prepare_kernel(prep, reinterpret_cast<const void*>(kern), C::kSmemBytes, &dev);
  if (rc != FA_OK) return rc;
  return launch_maybe_pdl(kern, grid, kQ4Threads, C::kSmemBytes, stream, pdl, mq, mk, mv, prm);
}

}  // namespace
}  // namespace fa

namespace fa {
namespace {
unsigned long long* g_trace_buffer = nullptr;
std::mutex g_ctr_mu;
unsigned int* g_ctr_base[64] = {};
int g_sm_count[64] = {};
std::atomic<unsigned int> g_ctr_next{0};

// Per device: the SM count and the counter pair of the next persistent
// launch.  A pair is reused after kUnitCtrSlots further launches; each launch
// leaves its pair at zero when its last CTA exits, and launches in one stream
// run in order, so a pair is never shared by two running launches unless
// kUnitCtrSlots launches were issued in between while the first still ran.
int persistent_setup(int dev, int* sms, unsigned int** ctr) {
  if (dev < 0 || dev >= 64) return FA_ERR_DEVICE;
  {
    std::lock_guard<std::mutex> lk(g_ctr_mu);
    if (g_ctr_base[dev] == nullptr) {
      void* a = nullptr;
      int n = 0;
      if (cudaGetSymbolAddress(&a, g_attn_unit_ctr) != cudaSuccess) return FA_ERR_CUDA;
      if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
          n <= 0)
        return FA_ERR_CUDA;
      g_ctr_base[dev] = static_cast<unsigned int*>(a);
      g_sm_count[dev] = n;
    }
  }
  *sms = g_sm_count[dev];
  *ctr = g_ctr_base[dev] + 2 * (g_ctr_next.fetch_add(1) % kUnitCtrSlots);
  return FA_OK;
}
}
}  // namespace fa

#ifdef FA_ATTN_TRACE
// Trace builds only: device buffer of kTraceCtas * kTraceIters * kTraceEvents
// 64-bit stamps that subsequent fa_attn_fwd launches fill.
extern "C" void fa_attn_set_trace_buffer(void* buf) {
  fa::g_trace_buffer = static_cast<unsigned long long*>(buf);
}
#endif

namespace fa {
namespace {

// Shared host path of fa_attn_fwd / fa_attn_fwd_f32 (arguments already
// validated): tensor maps, scheduling groups, launch.
// d_out: head dim of O when it differs from the operands' D (split mode:
// operand rows of 128 [hi | lo] values for a head dim <= 64).
int run_attn(const void* q, const void* k, const void* v, void* o, int B, int H, int S, int D,
             const int64_t* st, int causal, float scale, bool out_f32, bool f16,
             cudaStream_t stream, bool pdl = false, bool split = false, int d_out = 0) {
  int dev = 0;
  int rc = prepare_device(nullptr, 0, &dev);
  if (rc != FA_OK) return rc;
  // D <= 64: four-tile kernel with 64-key blocks; D <= 128: two-tile kernel.
  // Head dims below the kernel's width are zero-padded by the tensor maps.
  const bool q4 = (D <= 64) && !split;
  const int kv_rows = q4 ? kQ4BN : kBN;                  // keys per K/V block
  // Tiles per work unit: the kernel's width, halved while at most half the
  // SMs would get a unit (small problems spread over more SMs; a unit's
  // tiles share its K/V loads, so wide units stay where SMs are all busy).
  int sms = 0, tpu = q4 ? 4 : 2;
  unsigned int* ctr = nullptr;
  if ((rc = persistent_setup(dev, &sms, &ctr)) != FA_OK) return rc;
  while (tpu > 1 && 2 * static_cast<int64_t>(B) * H * ((S + tpu * kBM - 1) / (tpu * kBM)) <= sms)
    tpu /= 2;
  const int unit_rows = tpu * kBM;                         // query rows per unit
  CUtensorMap mq, mk, mv;
  if ((rc = make_tmap_bhsd(&mq, q, B, H, S, D, st[0], st[1], st[2], kBM, f16)) != FA_OK) return rc;
  if ((rc = make_tmap_bhsd(&mk, k, B, H, S, D, st[4], st[5], st[6], kv_rows, f16)) != FA_OK)
    return rc;
  if ((rc = make_tmap_bhsd(&mv, v, B, H, S, D, st[8], st[9], st[10], kv_rows, f16)) != FA_OK)
    return rc;

  AttnParams prm;
  prm.B = B;
  prm.H = H;
  prm.S = S;
  prm.D = d_out > 0 ? d_out : D;
  prm.n_units_per_head = (S + unit_rows - 1) / unit_rows;
  // Groups: at most FA_ATTN_GROUP_MIB of K/V each (>= 1 pair), the pairs
  // split as evenly as possible over them, since a short last group starts its
  // longest units late and leaves a tail.
  {
    const int64_t pairs = static_cast<int64_t>(B) * H;
    const int64_t kv_bytes_per_head = 2ll * S * D * 2;
    int64_t g = (static_cast<int64_t>(FA_ATTN_GROUP_MIB) << 20) /
                (kv_bytes_per_head > 0 ? kv_bytes_per_head : 1);
    if (g < 1) g = 1;
    if (g > pairs) g = pairs;
    const int64_t n_groups = (pairs + g - 1) / g;
    prm.group_q = static_cast<int>(pairs / n_groups);
    prm.group_r = static_cast<int>(pairs % n_groups);
  }
  prm.nkv = (S + kv_rows - 1) / kv_rows;
  prm.scale_log2 = scale * 1.4426950408889634f;
  prm.o = o;
  prm.o_sb = st[12];
  prm.o_sh = st[13];
  prm.o_ss = st[14];
  prm.status = device_status_ptr();
  prm.trace = g_trace_buffer;
  if (prm.status == nullptr) return FA_ERR_CUDA;
  int grid = static_cast<int>(static_cast<int64_t>(B) * H * prm.n_units_per_head);
  prm.total_units = grid;
  prm.unit_ctr = nullptr;
  prm.tiles_per_unit = tpu;
  prm.split_from = prm.total_units;
  if (FA_ATTN_PERSIST && grid > sms) {
    prm.unit_ctr = ctr;
    // Equal-length units (four-tile kernel, non-causal) leave a last partial
    // wave of r units on r SMs; when 2r SMs are available those units run
    // as 2r half units instead (B8 H16 S2048 D64: 512 units = 3 waves + 68).
    // Both halves of a split unit must hold rows: each head's last unit
    // (where the schedule ends) is full or more than half full.
    const int r = prm.total_units % sms;
    const int rem = S % unit_rows;
    if (FA_ATTN_SPLIT_TAIL && q4 && !causal && tpu == 4 && r > 0 && 2 * r <= sms &&
        (rem == 0 || 2 * rem > unit_rows)) {
      prm.split_from = prm.total_units - r;
      prm.total_units += r;
    }
    grid = sms;
  }
  if (q4) {
    if (out_f32)
      return causal ? launch_attn_q4<true, true, false>(mq, mk, mv, prm, grid, stream, pdl)
                    : launch_attn_q4<false, true, false>(mq, mk, mv, prm, grid, stream, pdl);
    if (f16)
      return causal ? launch_attn_q4<true, false, true>(mq, mk, mv, prm, grid, stream, pdl)
                    : launch_attn_q4<false, false, true>(mq, mk, mv, prm, grid, stream, pdl);
    return causal ? launch_attn_q4<true, false, false>(mq, mk, mv, prm, grid, stream, pdl)
                  : launch_attn_q4<false, false, false>(mq, mk, mv, prm, grid, stream, pdl);
  }
  if (split)
    return causal ? launch_attn<128, true, true, false, true>(mq, mk, mv, prm, grid, stream, pdl)
                  : launch_attn<128, false, true, false, true>(mq, mk, mv, prm, grid, stream,
                                                               pdl);
  if (out_f32)
    return causal ? launch_attn<128, true, true, false>(mq, mk, mv, prm, grid, stream, pdl)
                  : launch_attn<128, false, true, false>(mq, mk, mv, prm, grid, stream, pdl);
  if (f16)
    return causal ? launch_attn<128, true, false, true>(mq, mk, mv, prm, grid, stream, pdl)
                  : launch_attn<128, false, false, true>(mq, mk, mv, prm, grid, stream, pdl);
  return causal ? launch_attn<128, true, false, false>(mq, mk, mv, prm, grid, stream, pdl)
                : launch_attn<128, false, false, false>(mq, mk, mv, prm, grid, stream, pdl);
}

// fp32 -> bf16 staging of q, k, v (blockIdx.z picks the tensor) into the
// workspace [q | k | v].  Rows are the flattened (batch, head, position)
// index, S positions per (batch, head) matrix; K comes as [.., S, D] or, with
// k_transposed, as KT [.., D, S] (a 32 x 32 tile then goes through shared
// memory so reads and writes both stay coalesced).  split = 0: workspace
// rows of D bf16 values.  split = 1: rows of 128 values [hi | lo]: hi =
// bf16(x) in columns [0, D), lo = bf16(x - hi) in [64, 64 + D), zeros in the
// padding columns (the split-mode attention reads both 64-column atoms).
__global__ void __launch_bounds__(256)
    stage_f32_kernel(const float* __restrict__ q, const float* __restrict__ k,
                     const float* __restrict__ v, __nv_bfloat16* __restrict__ ws, int64_t rows,
                     int S, int D, int k_transposed, int split) {
  __shared__ float tile[32][33];
  // The attention kernel may start its set-up now; its loads wait for this
  // grid to complete.
  grid_dependents_launch();
  const int z = blockIdx.z;
  const float* src = (z == 0) ? q : (z == 1) ? k : v;
  const int W = split ? 128 : D;                       // workspace row width
  __nv_bfloat16* dst = ws + static_cast<int64_t>(z) * rows * W;
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * 32;
  const int d0 = blockIdx.y * 32;
  const int tx = threadIdx.x & 31;
  const int ty = threadIdx.x >> 5;   // 0..7
  // Value of element (row, d); zero outside the tensor.
  auto load = [&](int64_t row, int d) -> float {
    if (row >= rows || d >= D) return 0.f;
    if (z == 1 && k_transposed) {
      const int64_t bh = row / S, n = row - bh * S;
      return src[(bh * D + d) * S + n];
    }
    return src[row * D + d];
  };
  auto store = [&](int64_t row, int d, float x) {
    if (row >= rows) return;
    if (split) {
      const __nv_bfloat16 hi = __float2bfloat16_rn(x);
      dst[row * 128 + d] = hi;
      dst[row * 128 + 64 + d] = __float2bfloat16_rn(x - __bfloat162float(hi));
    } else if (d < D) {
      dst[row * D + d] = __float2bfloat16_rn(x);
    }
  };
  if (z == 1 && k_transposed) {
#pragma unroll
    for (int r = ty; r < 32; r += 8) tile[r][tx] = load(n0 + tx, d0 + r);   // read along n
    __syncthreads();
#pragma unroll
    for (int r = ty; r < 32; r += 8) store(n0 + r, d0 + tx, tile[tx][r]);   // write along d
  } else {
#pragma unroll
    for (int r = ty; r < 32; r += 8) store(n0 + r, d0 + tx, load(n0 + r, d0 + tx));
  }
}

// Self test of the softmax's exponentials on the device: for each x,
// out[i] = exp2_fma(x), out[n + i] = exp2_fma_x2 on the pair containing x,
// out[2n + i] = ex2.approx(x) -- the routines the attention kernels call.
__global__ void __launch_bounds__(256)
    exp2_selftest_kernel(const float* __restrict__ x, float* __restrict__ out, int n) {
  const int i = 2 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (i >= n) return;
  const float x0 = x[i];
  const float x1 = (i + 1 < n) ? x[i + 1] : 0.f;
  float a0, a1;
  exp2_fma_x2(x0, x1, a0, a1);
  out[i] = exp2_fma(x0);
  out[n + i] = a0;
  out[2 * n + i] = ex2_approx(x0);
  if (i + 1 < n) {
    out[i + 1] = exp2_fma(x1);
    out[n + i + 1] = a1;
    out[2 * n + i + 1] = ex2_approx(x1);
  }
}

}  // namespace
}  // namespace fa

extern "C" int fa_selftest_exp2(const float* x, float* out, int n, void* stream) {
  using namespace fa;
  if (!x || !out) return FA_ERR_NULL;
  if (n <= 0 || n > (1 << 28)) return FA_ERR_SHAPE;
  int dev = 0;
  const int rc = prepare_device(nullptr, 0, &dev);
  if (rc != FA_OK) return rc;
  const int threads = 256;
  const int blocks = ((n + 1) / 2 + threads - 1) / threads;
  exp2_selftest_kernel<<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(x, out, n);
  return cudaGetLastError() == cudaSuccess ? FA_OK : FA_ERR_LAUNCH;
}

namespace fa {
namespace {

bool head_dim_ok(int D) { return D >= 8 && D <= 128 && (D % 8) == 0; }

// Argument checks shared by fa_attn_fwd and fa_attn_fwd_f16 (no CUDA call).
int check_attn_args(const void* q, const void* k, const void* v, const void* o, int B, int H,
                    int S, int D, const int64_t* st) {
  if (!q || !k || !v || !o || !st) return FA_ERR_NULL;
  if (B <= 0 || H <= 0 || S <= 0) return FA_ERR_SHAPE;
  if (!head_dim_ok(D)) return FA_ERR_HEAD_DIM;
  const int64_t units = static_cast<int64_t>(B) * H * ((S + kBM - 1) / kBM);
  if (units > 0x7fffffffLL) return FA_ERR_SHAPE;
  for (int t = 0; t < 4; ++t) {
    if (st[4 * t + 3] != 1) return FA_ERR_STRIDE;
    for (int i = 0; i < 3; ++i)
      if (st[4 * t + i] <= 0 || (st[4 * t + i] % 8) != 0) return FA_ERR_ALIGN;
  }
  const void* ptrs[4] = {q, k, v, o};
  for (int t = 0; t < 4; ++t)
    if (reinterpret_cast<uintptr_t>(ptrs[t]) % 16 != 0) return FA_ERR_ALIGN;
  return FA_OK;
}

// fp32 -> bf16 staging of the B * H * S rows of each tensor into ws (split:
// [hi | lo] rows of 128 values), then the attention with an fp32 epilogue,
// launched as a programmatic dependent of the staging kernel.
int run_attn_f32(const void* q, const void* k, const void* v, void* o, void* ws, int B, int H,
                 int S, int D, int k_transposed, int causal, float scale, bool split,
                 cudaStream_t s) {
  int dev = 0;
  int rc = prepare_device(nullptr, 0, &dev);
  if (rc != FA_OK) return rc;
  __nv_bfloat16* wb = static_cast<__nv_bfloat16*>(ws);
  const int64_t rows = static_cast<int64_t>(B) * H * S;
  const int W = split ? 128 : D;
  const dim3 grid(static_cast<unsigned>((rows + 31) / 32), split ? 2 : (D + 31) / 32, 3);
  stage_f32_kernel<<<grid, 256, 0, s>>>(static_cast<const float*>(q),
                                       static_cast<const float*>(k),
                                       static_cast<const float*>(v), wb, rows, S, D, k_transposed,
                                       split ? 1 : 0);
  if (cudaGetLastError() != cudaSuccess) return FA_ERR_LAUNCH;
  const int64_t n = rows * W;
  const int64_t sw = static_cast<int64_t>(S) * W, hsw = sw * H;
  const int64_t so = static_cast<int64_t>(S) * D, hso = so * H;   // O: fp32 [B, H, S, D]
  const int64_t st[16] = {hsw, sw, W, 1, hsw, sw, W, 1, hsw, sw, W, 1, hso, so, D, 1};
  return run_attn(wb, wb + n, wb + 2 * n, o, B, H, S, W, st, causal, scale, true, false, s,
                  /*pdl=*/true, split, D);
}

}  // namespace
}  // namespace fa

extern "C" int fa_attn_fwd(const void* q, const void* k, const void* v, void* o, int B, int H,
                           int S, int D, const int64_t* st, int causal, float scale,
                           void* stream) {
  using namespace fa;
  const int rc = check_attn_args(q, k, v, o, B, H, S, D, st);
  if (rc != FA_OK) return rc;
  return run_attn(q, k, v, o, B, H, S, D, st, causal, scale, false, false,
                  static_cast<cudaStream_t>(stream));
}

extern "C" int fa_attn_fwd_f16(const void* q, const void* k, const void* v, void* o, int B,
                               int H, int S, int D, const int64_t* st, int causal, float scale,
                               void* stream) {
  using namespace fa;
  const int rc = check_attn_args(q, k, v, o, B, H, S, D, st);
  if (rc != FA_OK) return rc;
  return run_attn(q, k, v, o, B, H, S, D, st, causal, scale, false, true,
                  static_cast<cudaStream_t>(stream));
}

extern "C" int fa_attn_fwd_f32(const void* q, const void* k, const void* v, void* o, void* ws,
                               int N, int D, int k_transposed, int causal, float scale,
                               void* stream) {
  using namespace fa;
  if (!q || !k || !v || !o || !ws) return FA_ERR_NULL;
  if (N <= 0 || (k_transposed != 0 && k_transposed != 1)) return FA_ERR_SHAPE;
  if (!head_dim_ok(D)) return FA_ERR_HEAD_DIM;
  if (static_cast<int64_t>(N) * D > (1ll << 28)) return FA_ERR_SHAPE;
  const void* ptrs[5] = {q, k, v, o, ws};
  for (int t = 0; t < 5; ++t)
    if (reinterpret_cast<uintptr_t>(ptrs[t]) % 16 != 0) return FA_ERR_ALIGN;
  return run_attn_f32(q, k, v, o, ws, 1, 1, N, D, k_transposed, causal, scale, false,
                      static_cast<cudaStream_t>(stream));
}

extern "C" int fa_attn_fwd_f32_batched(const void* q, const void* k, const void* v, void* o,
                                       void* ws, int B, int H, int S, int D, int k_transposed,
                                       int causal, float scale, int precision, void* stream) {
  using namespace fa;
  if (!q || !k || !v || !o || !ws) return FA_ERR_NULL;
  if (B <= 0 || H <= 0 || S <= 0 || (k_transposed != 0 && k_transposed != 1)) return FA_ERR_SHAPE;
  if (precision != FA_F32_BF16 && precision != FA_F32_SPLIT) return FA_ERR_ARG;
  if (!head_dim_ok(D) || (precision == FA_F32_SPLIT && D > 64)) return FA_ERR_HEAD_DIM;
  const int64_t rows = static_cast<int64_t>(B) * H * S;
  if (rows * 128 > (1ll << 34) || (rows + 31) / 32 > 0x7fffffffLL ||
      static_cast<int64_t>(B) * H * ((S + kBM - 1) / kBM) > 0x7fffffffLL)
    return FA_ERR_SHAPE;
  const void* ptrs[5] = {q, k, v, o, ws};
  for (int t = 0; t < 5; ++t)
    if (reinterpret_cast<uintptr_t>(ptrs[t]) % 16 != 0) return FA_ERR_ALIGN;
  return run_attn_f32(q, k, v, o, ws, B, H, S, D, k_transposed, causal, scale,
                      precision == FA_F32_SPLIT, static_cast<cudaStream_t>(stream));
}
