// Causal paged prefill on tcgen05 tensor cores (sm_100a).
//
// One CTA (one per SM) owns two 128-row query tiles A and B of the same
// (sequence, KV head): tile A = tokens [t0, t0+tpt), tile B = the next tpt
// tokens; a row = (token, one of the G = Hq/Hkv query heads of the group), so
// every K/V tile loaded feeds 2 x 128 query rows. Keys stream in tiles of 128
// (eight 16-token blocks found through the block table): K through a 3-stage
// and V through a 2-stage shared-memory ring that both query tiles read.
//
//   warp 8 (TMA)    : Q_A, Q_B once (3-D boxes: 64 dims x G heads x tpt tokens,
//                     128B swizzle); then K_j, V_j per key tile (64-column boxes),
//                     K running one tile ahead of V.
//   warp 9 (MMA)    : one elected lane of a converged warp issues tcgen05.mma
//                     (kind::f16, fp32 accumulators in TMEM):
//                       S_X(j) = Q_X K_j^T  (M128 N128, 8 x K16; A, B K-major in smem)
//                       O_X   += P_X(j) V_j (M128 N128, 8 x K16; A = P_X in TMEM,
//                                            B = V_j MN-major in smem)
//                     in the order S_A(j), PV_B(j-1), S_B(j), PV_A(j): the softmax
//                     of one tile runs while the tensor core works on the other.
//   warps 0-3 / 4-7 : softmax of tile A / B; thread = TMEM lane = row:
//                     tcgen05.ld of the row's 128 scores, causal mask on diagonal
//                     key tiles only, online softmax in the log2 domain (scale
//                     folded into one packed FFMA, ex2.approx), P_X(j) (bf16/f16)
//                     written with tcgen05.st over the first 64 columns of S_X,
//                     O_X rescaled in TMEM only when a row max grows by > 2^8,
//                     O_X / l stored at the end.
//
// TMEM: S_A, S_B, O_A, O_B, 128 columns each = 512 (P_X aliased into S_X).
// Ordering: tcgen05.mma operations of one thread execute in issue order, and a
// commit arrives only when every earlier operation of the thread is complete.
// So S_X(j+1), issued after PV_X(j), overwrites P_X(j) only after it was read;
// and when the softmax sees S_X(j) complete, PV_X(j-1) is complete too, so it
// may rescale O_X without another wait.
// Barrier phases: every barrier completes at most once per key tile, and each
// waiter is at most one phase behind (S_X(j+1) needs P_X(j), which needs the
// softmax to have seen S_X(j)), so parity waits never alias.
// All waits are bounded; a timeout sets PS_DEVERR_TIMEOUT and a shared abort
// flag so every role leaves its loop, drains its in-flight copies / MMAs and
// frees TMEM before the CTA exits.
#include <algorithm>
#include <mutex>
#include <type_traits>

#include "capi_internal.h"
#include "common.cuh"
#include "tcgen05.cuh"

namespace ps {
namespace {

constexpr int kM = 128;   // query rows per query tile
constexpr int kN = 128;   // keys per KV tile
constexpr int kQHalf = kM * 128;   // one 64-column (128 B) slice of a Q tile: [128 rows][128 B]
constexpr int kKVHalf = kN * 128;  // one 64-column slice of a K or V tile: [128 keys][128 B]

// Layout for head dimension D (64 or 128): tiles are D/64 column slices of
// 128 B rows (one 128-byte swizzle atom wide). A smaller D leaves room for
// deeper K and V rings.
template <int D>
struct Cfg {
  static_assert(D == 64 || D == 128, "head_dim 64 or 128");
  static constexpr int kHalves = D / 64;
  static constexpr int kQBytes = kHalves * kQHalf;    // per query tile
  static constexpr int kKVBytes = kHalves * kKVHalf;  // K or V of one key tile
  static constexpr int kKStages = D == 64 ? 6 : 3;
  static constexpr int kVStages = D == 64 ? 5 : 2;
  static constexpr int kOffQ = 0;  // Q_A, Q_B
  static constexpr int kOffK = 2 * kQBytes;
  static constexpr int kOffV = kOffK + kKStages * kKVBytes;
  static constexpr int kOffBars = kOffV + kVStages * kKVBytes;
  static constexpr int kBarQ = 0;
  static constexpr int kBarKFull = 1;                       // [kKStages]
  static constexpr int kBarKEmpty = kBarKFull + kKStages;   // [kKStages]
  static constexpr int kBarVFull = kBarKEmpty + kKStages;   // [kVStages]
  static constexpr int kBarVEmpty = kBarVFull + kVStages;   // [kVStages]
  static constexpr int kBarSFull = kBarVEmpty + kVStages;   // [tile]
  static constexpr int kBarP = kBarSFull + 2;               // [tile]: P_X(j) written (128 arrivals)
  static constexpr int kBarOFinal = kBarP + 2;              // [tile]: the last PV of an item's tile
  static constexpr int kBarQFree = kBarOFinal + 2;          // an item's last S MMAs read Q_A, Q_B
  static constexpr int kBarDone = kBarQFree + 1;
  static constexpr int kNumBars = kBarDone + 1;
  static constexpr int kOffMisc = kOffBars + kNumBars * 8;  // [0] TMEM base, [1] abort flag
  static constexpr size_t kSmemBytes = 1024 + kOffMisc + 16;
  static_assert(kSmemBytes <= 232448, "exceeds the per-block shared memory limit");
};

// 12 warps = 3 warpgroups: softmax of tile A (warps 0-3), of tile B (4-7), and
// TMA (8) + MMA (9) + two idle warps. Registers are moved from the third
// warpgroup to the softmax ones with setmaxnreg: 256 x 192 + 128 x 64 = 57,344
// must not exceed the launch allocation (384 threads x the kernel's register
// count, 168), which the host checks before every launch. 192 for the softmax
// measured as fast as 216 (bit-identical output) and leaves ptxas no spills in
// any role; from 208 up it spills in the 64-register roles.
constexpr int kThreads = 384;
constexpr int kWarpTma = 8;
constexpr int kWarpMma = 9;
constexpr uint32_t kRegsSoftmax = 192;
constexpr uint32_t kRegsOther = 64;
constexpr int kRegPoolNeeded = 256 * kRegsSoftmax + 128 * kRegsOther;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemS = 0;    // S_X at X * 128 (P_X in its first 64 columns)
constexpr uint32_t kTmemO = 256;  // O_X at kTmemO + X * D
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale O only past 2^8 growth

struct PrefillParams {
  void* out;
  int64_t out_stride;
  const int32_t* block_tables;
  int64_t bt_stride;
  const int32_t* q_starts;
  const int32_t* q_lens;
  const int32_t* ctx_lens;
  int64_t num_blocks;
  int64_t num_rows;
  int num_kv_heads;
  int num_q_heads;
  int group;
  int tokens_per_tile;
  int max_blocks;
  int block_size;  // tokens per KV block: 8, 16 or 32
  int num_seqs;
  int num_q_tiles;  // query-tile pairs per sequence (of the longest)
  int num_items;    // num_q_tiles * num_kv_heads * num_seqs
  // Split-K over the key range: unit u = piece u % splits of item u / splits,
  // covering key tiles [piece * split_tiles, (piece + 1) * split_tiles). An
  // item longer than one piece writes unnormalised partials, merged by
  // prefill_combine_kernel; splits == 1 runs every item whole.
  int splits;
  int split_tiles;
  int num_units;     // num_items * splits
  float* part_o;     // [num_units][2 tiles][128 rows][D] fp32
  float2* part_ml;   // [num_units][2 tiles][128 rows] (running max, log2 units; row sum)
  float scale_log2;
  int32_t* err;
};

// One unit of work: two query tiles (tokens [t0, t0 + 2*tpt)) of one (sequence,
// KV head). Items are numbered group-major: the num_q_tiles items of one
// (sequence, KV head) are consecutive, so the static round-robin hands them to
// neighbouring CTAs of the same wave, and the K/V tiles they all read (the
// suffix is re-read by every later query tile) come from L2 instead of HBM.
// Inside a group the query tiles rotate by the wave the group starts in, so
// over the waves every CTA gets a mix of cheap (early) and expensive (late)
// tiles.
struct Item {
  int b, h, t0, q_len, ctx, q_start, ntiles, nblk_seq, last_key;
  int unit, j0;  // the unit, and its first key tile (0 unless split)
  bool partial;  // the item spans several pieces: write partials, not the output
};

// False when the unit has no rows or no keys (or invalid lengths, which set an
// error bit); every role decides identically from the same inputs. kSplit:
// the launch cuts items into key-range pieces (p.splits > 1); split items keep
// the most expensive query tile first inside a group, without the rotation
// (their pieces, not their tiles, spread the work). The unsplit kernel is its
// own instantiation, so none of the piece arithmetic reaches its loops
// (measured 5% slower on the prefix workload when it did).
template <bool kSplit>
__device__ __forceinline__ bool decode_item(const PrefillParams& p, int u, Item& w, bool report) {
  int it = u, piece = 0;
  if constexpr (kSplit) {
    it = u / p.splits;
    piece = u - it * p.splits;
  }
  const int nq = p.num_q_tiles;
  const int g = it / nq;                  // (sequence, KV head) group
  const int wave = kSplit ? 0 : (it - it % nq) / static_cast<int>(gridDim.x);  // wave the group starts in
  const int qt = nq - 1 - (it % nq + wave) % nq;
  w.b = g / p.num_kv_heads;
  w.h = g % p.num_kv_heads;
  w.q_len = p.q_lens[w.b];
  w.t0 = qt * 2 * p.tokens_per_tile;
  if (w.t0 >= w.q_len) return false;
  w.ctx = p.ctx_lens[w.b];
  w.q_start = p.q_starts[w.b];
  const int total = w.ctx + w.q_len;
  if (w.ctx < 0 || w.q_start < 0 || static_cast<int64_t>(w.q_start) + w.q_len > p.num_rows ||
      total > p.max_blocks * p.block_size) {
    if (report) set_device_error(p.err, PS_DEVERR_LENGTH);
    return false;
  }
  const int rows_here = min(2 * p.tokens_per_tile, w.q_len - w.t0);
  w.last_key = w.ctx + w.t0 + rows_here;  // keys [0, last_key) are needed
  const int item_tiles = (w.last_key + kN - 1) / kN;
  w.unit = u;
  if constexpr (kSplit) {
    w.j0 = piece * p.split_tiles;
    if (w.j0 >= item_tiles) return false;
    w.ntiles = min(p.split_tiles, item_tiles - w.j0);
    w.partial = item_tiles > p.split_tiles;
  } else {
    w.j0 = 0;
    w.ntiles = item_tiles;
    w.partial = false;
  }
  w.nblk_seq = (total + p.block_size - 1) / p.block_size;
  return true;
}

// Bounded mbarrier wait that also gives up when another role aborted. Inline:
// an out-of-line call here made ptxas fail register allocation in the softmax
// warpgroup.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort,
                                              int32_t* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t deadline = globaltimer_ns() + kWaitLimitNs;
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 0 && *abort) return false;
    if (globaltimer_ns() >= deadline) break;
  }
  *abort = 1;
  set_device_error(err, PS_DEVERR_TIMEOUT);
  return false;
}

// Bounded wait for the drains after a role's last item (TMA producer, MMA
// issuer), with the timed loop out of line. Measured on the 64-sequence
// prefix-prefill workload: 0.668 ms per launch against 0.681 ms with these
// waits inline too (same output bits); the call only costs the 64-register
// roles some spill traffic outside their loops.
static __device__ __noinline__ bool drain_wait_timed(uint64_t* bar, uint32_t parity) {
  const uint64_t deadline = globaltimer_ns() + kWaitLimitNs;
  do {
    if (mbar_try_wait(bar, parity)) return true;
  } while (globaltimer_ns() < deadline);
  return false;
}

__device__ __forceinline__ bool drain_wait(uint64_t* bar, uint32_t parity) {
  return mbar_try_wait(bar, parity) || drain_wait_timed(bar, parity);
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// max(a, b, c) in one instruction.
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// kind::f16 with the A operand in TMEM: D[tmem] (+)= A[tmem] * B[smem].
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(
          d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

// Softmax + epilogue of one query tile; 128 threads, thread = TMEM lane = row.
// g0: tiles this CTA processed before the item (S and P barrier phases);
// n: items before it (O barrier phase). Returns false once aborted.
template <typename T, int D, bool kSplit>
__device__ __forceinline__ bool softmax_tile(const PrefillParams& p, uint64_t* bars,
                                             volatile int* abort, uint32_t tmem, int tile, int r,
                                             int warp_in_tile, const Item& w, int g0, int n) {
  using C = Cfg<D>;
  const int ntiles = w.ntiles;
  const int t0_tile = w.t0 + tile * p.tokens_per_tile;
  const int ctx = w.ctx, q_len = w.q_len, q_start = w.q_start, h = w.h, last_key = w.last_key;
  const int G = p.group;
  const int tpt = p.tokens_per_tile;
  const int tok = r / G;
  const bool row_real = (r < G * tpt) && (t0_tile + tok < q_len);
  const int limit = row_real ? ctx + t0_tile + tok : last_key - 1;  // last key this row sees
  const int tile_min_limit = ctx + t0_tile;  // smallest limit among this tile's real rows
  const uint32_t lane_tmem = tmem + (static_cast<uint32_t>(warp_in_tile * 32) << 16);
  const uint32_t s_col = kTmemS + tile * kN;
  const uint32_t o_col = kTmemO + tile * D;
  const float2 scale2 = make_float2(p.scale_log2, p.scale_log2);
  float m_used = -INFINITY;  // running max, log2-scaled
  float l_sum = 0.f;
  bool ok = true;
  for (int j = 0; j < ntiles; ++j) {
    ok = wait_or_abort(&bars[C::kBarSFull + tile], (g0 + j) & 1, abort, p.err);
    ok = __all_sync(0xffffffffu, ok);
    if (!ok) break;
    tc_fence_after();
    uint32_t sraw[4][32];
#pragma unroll
    for (int c = 0; c < 4; ++c) tmem_ld32(lane_tmem + s_col + c * 32, sraw[c]);
    tmem_wait_ld();
    float* s = reinterpret_cast<float*>(&sraw[0][0]);
    const int key0 = (w.j0 + j) * kN;
    if (key0 + kN - 1 > tile_min_limit) {  // diagonal tile: causal mask (warp-uniform test)
#pragma unroll
      for (int c = 0; c < kN; ++c)
        if (key0 + c > limit) s[c] = -INFINITY;
    }
    // Row max on four chains: s[0..3], then 3-input steps over s[4..kN-5], then
    // the last four scores (kN - 4 is not a multiple of 8).
    static_assert(kN % 8 == 0, "the row max walks the scores in groups of 8");
    float mx[4] = {s[0], s[1], s[2], s[3]};
#pragma unroll
    for (int c = 4; c + 8 <= kN; c += 8) {
#pragma unroll
      for (int e = 0; e < 4; ++e) mx[e] = max3f(mx[e], s[c + e], s[c + 4 + e]);
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) mx[e] = fmaxf(mx[e], s[kN - 4 + e]);
    const float mt = max3f(mx[0], mx[1], fmaxf(mx[2], mx[3])) * p.scale_log2;
    const bool rescale = __any_sync(0xffffffffu, mt > m_used + kRescaleThreshold);
    float alpha = 1.f;
    if (rescale) {
      const float m_new = fmaxf(m_used, mt);
      alpha = (m_new == -INFINITY) ? 1.f : ex2_approx(m_used - m_new);
      m_used = m_new;
    }
    // p = 2^(s*scale - m) -> P_X(j) as packed pairs (lane r = row r) over the
    // first 64 columns of S_X, 16 columns at a time. The row sum adds the fp32
    // exponentials: summing the rounded P after P is handed over measured 4.8%
    // slower with the same error against the fp32 oracle.
    // A row with no key yet (only in a piece past its causal limit) keeps
    // m_used = -inf; its masked scores give 2^-inf = 0 against 0.
    float m_exp = m_used;
    if constexpr (kSplit) m_exp = m_used == -INFINITY ? 0.f : m_used;
    const float2 negm = make_float2(-m_exp, -m_exp);
    float2 ls[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                    make_float2(0.f, 0.f)};  // four independent add chains
#pragma unroll
    for (int c = 0; c < kN; c += 32) {
      uint32_t packed[16];
#pragma unroll
      for (int e = 0; e < 32; e += 2) {
        const float2 x = __ffma2_rn(make_float2(s[c + e], s[c + e + 1]), scale2, negm);
        const float2 pe = make_float2(ex2_approx(x.x), ex2_approx(x.y));
        packed[e >> 1] = pack2<T>(pe);
        ls[(e >> 1) & 3] = __fadd2_rn(ls[(e >> 1) & 3], pe);
      }
      tmem_st16(lane_tmem + s_col + (c >> 1), packed);
    }
    const float2 ls01 = __fadd2_rn(ls[0], ls[1]);
    const float2 ls23 = __fadd2_rn(ls[2], ls[3]);
    l_sum = l_sum * alpha + ((ls01.x + ls23.x) + (ls01.y + ls23.y));
    if (rescale && j > 0) {
      // After the scores are consumed (fewer live registers); before P_X(j) is
      // announced, so PV_X(j) accumulates into the rescaled O_X. S_X(j)
      // complete implies PV_X(j-1) complete: O_X is stable here.
      const float2 a2 = make_float2(alpha, alpha);
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(lane_tmem + o_col + c * 32, o);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const float2 v =
              __fmul2_rn(make_float2(__uint_as_float(o[e]), __uint_as_float(o[e + 1])), a2);
          o[e] = __float_as_uint(v.x);
          o[e + 1] = __float_as_uint(v.y);
        }
        tmem_st32(lane_tmem + o_col + c * 32, o);
      }
    }
    tmem_wait_st();
    tc_fence_before();
    mbar_arrive(&bars[C::kBarP + tile]);
  }
  if (ok) {
    ok = wait_or_abort(&bars[C::kBarOFinal + tile], n & 1, abort, p.err);
    ok = __all_sync(0xffffffffu, ok);
  }
  if (!ok) return false;
  tc_fence_after();
  if (kSplit && w.partial) {
    // One piece of a split item: unnormalised O with its running max and row
    // sum, for prefill_combine_kernel.
    uint32_t oall[D / 32][32];
#pragma unroll
    for (int c = 0; c < D / 32; ++c) tmem_ld32(lane_tmem + o_col + c * 32, oall[c]);
    tmem_wait_ld();
    if (row_real) {
      const int64_t prow = (static_cast<int64_t>(w.unit) * 2 + tile) * kM + r;
      float4* po = reinterpret_cast<float4*>(p.part_o + prow * D);
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
#pragma unroll
        for (int v = 0; v < 8; ++v)
          po[c * 8 + v] = make_float4(__uint_as_float(oall[c][4 * v]), __uint_as_float(oall[c][4 * v + 1]),
                                      __uint_as_float(oall[c][4 * v + 2]), __uint_as_float(oall[c][4 * v + 3]));
      }
      p.part_ml[prow] = make_float2(m_used, l_sum);
    }
    tc_fence_before();
    return true;
  }
  const float inv = (l_sum > 0.f) ? 1.f / l_sum : 0.f;
  const int64_t out_row = static_cast<int64_t>(q_start) + t0_tile + tok;
  T* orow = static_cast<T*>(p.out) + out_row * p.out_stride +
            static_cast<int64_t>(h * G + (r % G)) * D;
  // The whole row in one TMEM round trip (four loads, one wait): measured
  // 0.5-0.7% faster per launch than a wait after every 32 columns.
  uint32_t oall[D / 32][32];
#pragma unroll
  for (int c = 0; c < D / 32; ++c) tmem_ld32(lane_tmem + o_col + c * 32, oall[c]);
  tmem_wait_ld();
  if (row_real) {
#pragma unroll
    for (int c = 0; c < D / 32; ++c) {
      const uint32_t* o = oall[c];
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        uint4 st;
        st.x = pack2<T>(__uint_as_float(o[8 * v + 0]) * inv, __uint_as_float(o[8 * v + 1]) * inv);
        st.y = pack2<T>(__uint_as_float(o[8 * v + 2]) * inv, __uint_as_float(o[8 * v + 3]) * inv);
        st.z = pack2<T>(__uint_as_float(o[8 * v + 4]) * inv, __uint_as_float(o[8 * v + 5]) * inv);
        st.w = pack2<T>(__uint_as_float(o[8 * v + 6]) * inv, __uint_as_float(o[8 * v + 7]) * inv);
        *reinterpret_cast<uint4*>(orow + c * 32 + 8 * v) = st;
      }
    }
  }
  // This item's O_X has been read out: the next item's first PV may overwrite
  // it (its P_X arrives only after this point).
  tc_fence_before();
  return true;
}

// BS = tokens per KV block (8, 16 or 32): a 128-key tile is 128/BS block boxes.
template <typename T, int D, int BS, bool kSplit>
__global__ void __launch_bounds__(kThreads, 1)
    paged_prefill_kernel(const PrefillParams p, const __grid_constant__ CUtensorMap qmap,
                         const __grid_constant__ CUtensorMap kmap,
                         const __grid_constant__ CUtensorMap vmap) {
  using C = Cfg<D>;
  constexpr int kTileBlocks = kN / BS;
  static_assert(kTileBlocks <= 32, "one 32-lane window of block ids must cover a tile");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBars);
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + C::kOffMisc);
  volatile int* abort = reinterpret_cast<volatile int*>(misc + 1);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = p.group;
  const int tpt = p.tokens_per_tile;

  // Launched with programmatic stream serialization: barrier set-up and the
  // TMEM allocation overlap the previous kernel's end; global memory is
  // touched only after pdl_wait().
  pdl_trigger();
  if (threadIdx.x == 0) {
    for (int i = 0; i < C::kNumBars; ++i) mbar_init(&bars[i], (i >= C::kBarP && i < C::kBarP + 2) ? 128 : 1);
    *abort = 0;
    fence_barrier_init();
  }
  if (warp == kWarpMma) tmem_alloc(&misc[0], kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = misc[0];
  pdl_wait();

  // Persistent: CTA c takes items c, c + gridDim.x, ... Every role walks the
  // same items; ring positions and barrier phases carry over from item to item.
  // Branch per warpgroup first, so each register budget covers exactly its code.
  if (warp >= 8) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsOther));
  if (warp == kWarpTma) {
    // ------------------------------------------------------------ TMA producer
    // The whole warp walks the tiles so block ids arrive 32 at a time (one
    // coalesced load per 4 key tiles, shuffled to lane 0) instead of one L2
    // round trip per block; lane 0 issues every barrier op and TMA load.
    // Per item: K_0, then Q_A, Q_B once the previous item's last S MMAs are
    // done with them, then K_{j+1} before V_j, so K (needed first) runs ahead.
    if (lane == 0) {
      tma_prefetch_desc(&qmap);
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
    }
    int kc = 0, vc = 0, n = 0;  // K, V tiles and items issued so far
    bool ok = true;
    for (int it = blockIdx.x; ok && it < p.num_units; it += gridDim.x) {
      Item w;
      if (!decode_item<kSplit>(p, it, w, lane == 0)) continue;
      const int32_t* bt = p.block_tables + static_cast<int64_t>(w.b) * p.bt_stride;
      int window = -32;  // first block index held by the lanes' `my_row`
      int32_t my_row = 0;
      // Block-row coordinates of key tile j (uniform across the warp).
      auto tile_rows = [&](int j, int32_t (&rows)[kTileBlocks]) {
        const int kb0 = j * kTileBlocks;
        if (kb0 >= window + 32) {
          window = kb0;
          const int kb = window + lane;
          int32_t id = 0;
          if (kb < w.nblk_seq) {
            id = bt[kb];
            if (id < 0 || id >= p.num_blocks) {
              set_device_error(p.err, PS_DEVERR_BLOCK_ID);
              id = 0;
            }
          }
          my_row = kb < w.nblk_seq ? (id * p.num_kv_heads + w.h) * BS : -1;
        }
#pragma unroll
        for (int bb = 0; bb < kTileBlocks; ++bb)
          rows[bb] = __shfl_sync(0xffffffffu, my_row, kb0 - window + bb);
#pragma unroll
        for (int bb = 1; bb < kTileBlocks; ++bb)  // past the sequence end: re-read a valid block (masked)
          if (rows[bb] < 0) rows[bb] = rows[0];
      };
      // One K or V tile (global index g) into its ring stage (lane 0); false once aborted.
      auto load_tile = [&](const CUtensorMap* map, uint8_t* base, int full, int empty, int stages,
                           int g, const int32_t (&rows)[kTileBlocks]) -> bool {
        bool good = true;
        if (lane == 0) {
          const int st = g % stages;
          if (g >= stages)
            good = wait_or_abort(&bars[empty + st], ((g / stages) - 1) & 1, abort, p.err);
          if (good) {
            uint8_t* dst = base + st * C::kKVBytes;
            mbar_arrive_expect_tx(&bars[full + st], C::kKVBytes);
#pragma unroll
            for (int bb = 0; bb < kTileBlocks; ++bb) {
#pragma unroll
              for (int hh = 0; hh < C::kHalves; ++hh)
                tma_load_2d(dst + hh * kKVHalf + bb * (BS * 128), map, &bars[full + st],
                            64 * hh, rows[bb]);
            }
          }
        }
        return __shfl_sync(0xffffffffu, good ? 1 : 0, 0) != 0;
      };
      int32_t rows_k[kTileBlocks], rows_v[kTileBlocks];
      tile_rows(w.j0, rows_k);
      if (!(ok = load_tile(&kmap, smem + C::kOffK, C::kBarKFull, C::kBarKEmpty, C::kKStages, kc, rows_k)))
        break;
      ++kc;
      if (lane == 0) {
        if (n > 0) ok = wait_or_abort(&bars[C::kBarQFree], (n - 1) & 1, abort, p.err);
        if (ok) {
          mbar_arrive_expect_tx(&bars[C::kBarQ], 2u * C::kHalves * 64u * G * tpt * 2u);
#pragma unroll
          for (int x = 0; x < 2; ++x) {
            uint8_t* q = smem + C::kOffQ + x * C::kQBytes;
            const int row = w.q_start + w.t0 + x * tpt;
#pragma unroll
            for (int hh = 0; hh < C::kHalves; ++hh)
              tma_load_3d(q + hh * kQHalf, &qmap, &bars[C::kBarQ], 64 * hh, w.h * G, row);
          }
        }
      }
      if (!(ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0)) break;
      ++n;
      for (int j = 0; j < w.ntiles; ++j) {
#pragma unroll
        for (int bb = 0; bb < kTileBlocks; ++bb) rows_v[bb] = rows_k[bb];  // tile j's blocks
        if (j + 1 < w.ntiles) {
          tile_rows(w.j0 + j + 1, rows_k);
          if (!(ok = load_tile(&kmap, smem + C::kOffK, C::kBarKFull, C::kBarKEmpty, C::kKStages, kc, rows_k)))
            break;
          ++kc;
        }
        if (!(ok = load_tile(&vmap, smem + C::kOffV, C::kBarVFull, C::kBarVEmpty, C::kVStages, vc, rows_v)))
          break;
        ++vc;
      }
    }
    if (lane == 0) {
      // Drain: the last Q and the last load issued into each stage have landed.
      if (n > 0) (void)drain_wait(&bars[C::kBarQ], (n - 1) & 1);
      for (int g = max(0, kc - C::kKStages); g < kc; ++g)
        (void)drain_wait(&bars[C::kBarKFull + (g % C::kKStages)], (g / C::kKStages) & 1);
      for (int g = max(0, vc - C::kVStages); g < vc; ++g)
        (void)drain_wait(&bars[C::kBarVFull + (g % C::kVStages)], (g / C::kVStages) & 1);
    }
  } else if (warp == kWarpMma) {
    // ------------------------------------------------------------ MMA issuer
    // The whole warp runs this loop (waits, descriptor arithmetic: all
    // warp-uniform); one elected lane issues each tcgen05.mma / commit.
    const bool leader = elect_one();
    constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
    constexpr uint32_t kIdS = idesc_f16(kBf16, kM, kN, false, false);
    constexpr uint32_t kIdO = idesc_f16(kBf16, kM, D, false, true);
    // Descriptors are built once; stepping through K, stages and buffers only
    // adds (byte offset >> 4) to the start-address field (addresses < 256 KB,
    // so the 14-bit field never carries).
    const uint64_t q_desc = sdesc_sw128(smem_u32(smem + C::kOffQ), 16, 1024);
    const uint64_t k_desc = sdesc_sw128(smem_u32(smem + C::kOffK), 16, 1024);
    const uint64_t v_desc = sdesc_sw128(smem_u32(smem + C::kOffV), kKVHalf, 1024);
    auto wait_all = [&](uint64_t* bar, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, wait_or_abort(bar, parity, abort, p.err));
    };
    // S_X = Q_X K^T for the K tile with global index kg (its stage must be full).
    auto issue_s = [&](int x, int kg) {
      const uint64_t kd = k_desc + static_cast<uint64_t>(((kg % C::kKStages) * C::kKVBytes) >> 4);
      const uint32_t d = tmem + kTmemS + x * kN;
      const uint64_t qd = q_desc + static_cast<uint64_t>(x * (C::kQBytes >> 4));
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint32_t off = ((kk >> 2) * kQHalf + (kk & 3) * 32) >> 4;
        const uint32_t koff = ((kk >> 2) * kKVHalf + (kk & 3) * 32) >> 4;
        if (leader) umma_f16(d, qd + off, kd + koff, kIdS, kk > 0 ? 1u : 0u);
      }
      if (leader) umma_commit(&bars[C::kBarSFull + x]);
    };
    // O_X += P_X V for the V tile with global index vg (already waited for) once
    // the softmax of tile X has written P_X (its g-th).
    auto issue_pv = [&](int x, int g, int vg, bool first, bool last) -> bool {
      if (!wait_all(&bars[C::kBarP + x], g & 1)) return false;
      tc_fence_after();
      const uint64_t vd = v_desc + static_cast<uint64_t>(((vg % C::kVStages) * C::kKVBytes) >> 4);
      const uint32_t p_tmem = tmem + kTmemS + x * kN;
#pragma unroll
      for (int kk = 0; kk < kN / 16; ++kk) {
        if (leader)
          umma_f16_ts(tmem + kTmemO + x * D, p_tmem + kk * 8, vd + (kk * 2048 >> 4), kIdO,
                      (!first || kk > 0) ? 1u : 0u);
      }
      if (leader && last) umma_commit(&bars[C::kBarOFinal + x]);
      return true;
    };
    // The K and V waits are taken while the softmax of the tile is still running
    // (never between a P arrival and the MMAs it releases): K_j before S_A(j)
    // was waited one tile earlier, V_j before P_A(j) serves PV_A(j) and PV_B(j).
    int kc = 0, vc = 0, g = 0, n = 0;  // K, V tiles, S/P phases and items consumed so far
    bool ok = true;
    for (int it = blockIdx.x; ok && it < p.num_units; it += gridDim.x) {
      Item w;
      if (!decode_item<kSplit>(p, it, w, false)) continue;
      if (!(ok = wait_all(&bars[C::kBarQ], n & 1))) break;
      if (!(ok = wait_all(&bars[C::kBarKFull + kc % C::kKStages], (kc / C::kKStages) & 1))) break;
      tc_fence_after();
      const int nt = w.ntiles;
      for (int j = 0; j < nt; ++j) {
        issue_s(0, kc + j);
        if (j > 0) {
          if (!(ok = issue_pv(1, g + j - 1, vc + j - 1, j == 1, false))) break;
          if (leader) umma_commit(&bars[C::kBarVEmpty + (vc + j - 1) % C::kVStages]);
        }
        issue_s(1, kc + j);
        if (leader) {
          umma_commit(&bars[C::kBarKEmpty + (kc + j) % C::kKStages]);
          if (j + 1 == nt) umma_commit(&bars[C::kBarQFree]);
        }
        if (!(ok = wait_all(&bars[C::kBarVFull + (vc + j) % C::kVStages], ((vc + j) / C::kVStages) & 1)))
          break;
        if (j + 1 < nt &&
            !(ok = wait_all(&bars[C::kBarKFull + (kc + j + 1) % C::kKStages],
                            ((kc + j + 1) / C::kKStages) & 1)))
          break;
        if (!(ok = issue_pv(0, g + j, vc + j, j == 0, j + 1 == nt))) break;
      }
      if (!ok) break;
      if (!(ok = issue_pv(1, g + nt - 1, vc + nt - 1, nt == 1, true))) break;
      if (leader) umma_commit(&bars[C::kBarVEmpty + (vc + nt - 1) % C::kVStages]);
      kc += nt;
      vc += nt;
      g += nt;
      ++n;
    }
    // Every MMA issued above has completed before TMEM is released.
    if (leader) umma_commit(&bars[C::kBarDone]);
    __syncwarp();
    (void)drain_wait(&bars[C::kBarDone], 0);
  }  // warps 10 and 11 have no role
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));
    // ------------------------------------------------------------ softmax + epilogue
    const int x = warp >> 2;  // query tile 0 (A) or 1 (B)
    int g = 0, n = 0;
    for (int it = blockIdx.x; it < p.num_units; it += gridDim.x) {
      Item w;
      if (!decode_item<kSplit>(p, it, w, false)) continue;
      if (!softmax_tile<T, D, kSplit>(p, bars, abort, tmem, x, threadIdx.x & 127, warp & 3, w, g, n))
        break;
      g += w.ntiles;
      ++n;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// Merges the pieces of split items: one warp per (item, query tile, row), each
// lane D/32 columns. With m* the largest running max over the pieces and
// w_s = 2^(m_s - m*): out = sum_s w_s O_s / sum_s w_s l_s. Items that were not
// split, and rows past a sequence's new tokens, are left to the prefill kernel.
constexpr int kCombineWarps = 8;

template <typename T, int D>
__global__ void __launch_bounds__(kCombineWarps * 32)
    prefill_combine_kernel(const PrefillParams p) {
  pdl_wait();
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * kCombineWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int it = static_cast<int>(gw / (2 * kM));
  if (it >= p.num_items) return;
  const int tile = static_cast<int>(gw % (2 * kM)) / kM;
  const int r = static_cast<int>(gw % kM);
  Item w;
  if (!decode_item<true>(p, it * p.splits, w, false) || !w.partial) return;
  const int G = p.group;
  const int t0_tile = w.t0 + tile * p.tokens_per_tile;
  const int tok = r / G;
  if (r >= G * p.tokens_per_tile || t0_tile + tok >= w.q_len) return;
  const int item_tiles = (w.last_key + kN - 1) / kN;
  const int pieces = (item_tiles + p.split_tiles - 1) / p.split_tiles;
  const int64_t row0 = (static_cast<int64_t>(it) * p.splits * 2 + tile) * kM + r;
  const int64_t piece_stride = 2 * kM;  // rows between consecutive pieces of the item
  float m_star = -INFINITY;
  for (int s = 0; s < pieces; ++s) m_star = fmaxf(m_star, p.part_ml[row0 + s * piece_stride].x);
  constexpr int V = D / 32;
  float acc[V] = {};
  float l_tot = 0.f;
  for (int s = 0; s < pieces; ++s) {
    const int64_t row = row0 + s * piece_stride;
    const float2 ml = p.part_ml[row];
    const float wgt = ml.x == -INFINITY ? 0.f : ex2_approx(ml.x - m_star);
    l_tot += wgt * ml.y;
    const float* o = p.part_o + row * D + lane * V;
    if constexpr (V == 4) {
      const float4 v = *reinterpret_cast<const float4*>(o);
      acc[0] += wgt * v.x; acc[1] += wgt * v.y; acc[2] += wgt * v.z; acc[3] += wgt * v.w;
    } else {
      const float2 v = *reinterpret_cast<const float2*>(o);
      acc[0] += wgt * v.x; acc[1] += wgt * v.y;
    }
  }
  const float inv = l_tot > 0.f ? 1.f / l_tot : 0.f;
  const int64_t out_row = static_cast<int64_t>(w.q_start) + t0_tile + tok;
  T* orow = static_cast<T*>(p.out) + out_row * p.out_stride +
            static_cast<int64_t>(w.h * G + (r % G)) * D + lane * V;
  if constexpr (V == 4) {
    uint2 st;
    st.x = pack2<T>(acc[0] * inv, acc[1] * inv);
    st.y = pack2<T>(acc[2] * inv, acc[3] * inv);
    *reinterpret_cast<uint2*>(orow) = st;
  } else {
    *reinterpret_cast<uint32_t*>(orow) = pack2<T>(acc[0] * inv, acc[1] * inv);
  }
}

// One per element type: the dynamic shared-memory opt-in is per kernel and per device.
template <typename T, int D, int BS, bool kSplit>
int launch_prefill(const PrefillParams& p, const CUtensorMap& qm, const CUtensorMap& km,
                   const CUtensorMap& vm, dim3 grid, cudaStream_t s) {
  static bool configured[64] = {};
  static std::mutex mu;  // concurrent host threads
  std::unique_lock<std::mutex> lock(mu);
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    // setmaxnreg.inc waits until the pool holds the registers it asks for: a
    // split above the launch allocation would never proceed, so refuse it here.
    cudaFuncAttributes fa{};
    cudaError_t e = cudaFuncGetAttributes(&fa, paged_prefill_kernel<T, D, BS, kSplit>);
    if (e != cudaSuccess)
      return fail(PS_ERR_CUDA, "ps_paged_prefill: cannot read kernel attributes: %s",
                  cudaGetErrorString(e));
    if (fa.numRegs * kThreads < kRegPoolNeeded || fa.maxThreadsPerBlock < kThreads)
      return fail(PS_ERR_UNSUPPORTED,
                  "ps_paged_prefill: kernel built with %d registers x %d threads, the register "
                  "split needs %d",
                  fa.numRegs, kThreads, kRegPoolNeeded);
    e = cudaFuncSetAttribute(paged_prefill_kernel<T, D, BS, kSplit>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(Cfg<D>::kSmemBytes));
    if (e != cudaSuccess)
      return fail(PS_ERR_CUDA, "ps_paged_prefill: cannot reserve %zu B shared memory: %s",
                  Cfg<D>::kSmemBytes, cudaGetErrorString(e));
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  lock.unlock();
  cudaError_t e = launch_pdl(paged_prefill_kernel<T, D, BS, kSplit>, grid, dim3(kThreads),
                             Cfg<D>::kSmemBytes, s, p, qm, km, vm);
  if (e != cudaSuccess)
    return fail(PS_ERR_CUDA, "ps_paged_prefill: launch failed: %s", cudaGetErrorString(e));
  if (kSplit) {
    const int64_t warps = static_cast<int64_t>(p.num_items) * 2 * kM;
    const dim3 cgrid(static_cast<unsigned>((warps + kCombineWarps - 1) / kCombineWarps));
    e = launch_pdl(prefill_combine_kernel<T, D>, cgrid, dim3(kCombineWarps * 32), 0, s, p);
    if (e != cudaSuccess)
      return fail(PS_ERR_CUDA, "ps_paged_prefill: combine launch failed: %s",
                  cudaGetErrorString(e));
  }
  return check_launch("ps_paged_prefill");
}

template <typename T, int D>
int dispatch_bs(const PrefillParams& p, const CUtensorMap& qm, const CUtensorMap& km,
                const CUtensorMap& vm, dim3 grid, cudaStream_t s, int block_size) {
  const bool split = p.splits > 1;
  if (block_size == 8)
    return split ? launch_prefill<T, D, 8, true>(p, qm, km, vm, grid, s)
                 : launch_prefill<T, D, 8, false>(p, qm, km, vm, grid, s);
  if (block_size == 32)
    return split ? launch_prefill<T, D, 32, true>(p, qm, km, vm, grid, s)
                 : launch_prefill<T, D, 32, false>(p, qm, km, vm, grid, s);
  return split ? launch_prefill<T, D, 16, true>(p, qm, km, vm, grid, s)
               : launch_prefill<T, D, 16, false>(p, qm, km, vm, grid, s);
}

int dispatch_prefill(const PrefillParams& p, const CUtensorMap& qm, const CUtensorMap& km,
                     const CUtensorMap& vm, dim3 grid, cudaStream_t s, int dtype, int head_dim,
                     int block_size) {
  if (dtype == PS_DTYPE_BF16)
    return head_dim == 64 ? dispatch_bs<__nv_bfloat16, 64>(p, qm, km, vm, grid, s, block_size)
                          : dispatch_bs<__nv_bfloat16, 128>(p, qm, km, vm, grid, s, block_size);
  return head_dim == 64 ? dispatch_bs<__half, 64>(p, qm, km, vm, grid, s, block_size)
                        : dispatch_bs<__half, 128>(p, qm, km, vm, grid, s, block_size);
}

// Work-unit layout of a launch: items (query-tile pairs of one sequence and KV
// head), each cut into `splits` key-range pieces of split_tiles key tiles (one
// piece of "all of it" when split_keys is 0 or covers the longest context),
// and the workspace the pieces' partials need.
struct SplitGeometry {
  int64_t items = 0;
  int splits = 1;
  int split_tiles = 1 << 30;
  int64_t units = 0;
  int64_t o_bytes = 0;   // partial O, fp32
  int64_t ml_bytes = 0;  // running max and row sum per row
  int64_t workspace_bytes() const {
    return splits > 1 ? ((o_bytes + 255) / 256 + (ml_bytes + 255) / 256) * 256 : 0;
  }
};

SplitGeometry split_geometry(int num_seqs, int max_q_len, int group, int num_kv_heads,
                             int head_dim, int block_size, int max_blocks_per_seq,
                             int split_keys) {
  SplitGeometry g;
  const int tpt = kM / group;
  g.items = static_cast<int64_t>((max_q_len + 2 * tpt - 1) / (2 * tpt)) * num_kv_heads * num_seqs;
  const int64_t max_tiles = (static_cast<int64_t>(max_blocks_per_seq) * block_size + kN - 1) / kN;
  if (split_keys > 0 && max_tiles > split_keys / kN) {
    g.split_tiles = split_keys / kN;
    g.splits = static_cast<int>((max_tiles + g.split_tiles - 1) / g.split_tiles);
  }
  g.units = g.items * g.splits;
  g.o_bytes = g.units * 2 * kM * head_dim * 4;
  g.ml_bytes = g.units * 2 * kM * 8;
  return g;
}

int prefill_entry(const char* fn, void* out, int64_t out_token_stride, const void* query,
                  int64_t query_token_stride, int64_t num_query_rows, const void* k_pool,
                  const void* v_pool, int64_t num_blocks, const int32_t* block_tables,
                  int64_t block_table_stride, const int32_t* q_starts, const int32_t* q_lens,
                  const int32_t* ctx_lens, int num_seqs, int max_q_len, int num_q_heads,
                  int num_kv_heads, int head_dim, int block_size, int max_blocks_per_seq,
                  float scale, int split_keys, void* workspace, int64_t workspace_bytes,
                  int dtype, int32_t* device_error, void* stream) {
  if (dtype != PS_DTYPE_BF16 && dtype != PS_DTYPE_F16)
    return fail(PS_ERR_UNSUPPORTED, "%s: dtype %d unsupported (bf16/f16 only)", fn, dtype);
  if (head_dim != 64 && head_dim != 128)
    return fail(PS_ERR_UNSUPPORTED, "%s: head_dim %d unsupported (64 or 128)", fn, head_dim);
  if (block_size != 8 && block_size != 16 && block_size != 32)
    return fail(PS_ERR_UNSUPPORTED, "%s: block_size %d unsupported (8, 16 or 32)", fn,
                block_size);
  if (num_seqs < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || num_blocks <= 0 ||
      max_blocks_per_seq <= 0 || num_query_rows < 0 || max_q_len < 0)
    return fail(PS_ERR_INVALID, "%s: bad sizes", fn);
  if (num_q_heads % num_kv_heads != 0)
    return fail(PS_ERR_INVALID, "%s: num_q_heads %d not divisible by num_kv_heads %d", fn,
                num_q_heads, num_kv_heads);
  const int group = num_q_heads / num_kv_heads;
  if (group > 16)
    return fail(PS_ERR_UNSUPPORTED, "%s: %d query heads per kv head unsupported (max 16)", fn,
                group);
  if (split_keys < 0 || split_keys % kN)
    return fail(PS_ERR_INVALID, "%s: split_keys %d must be a non-negative multiple of %d", fn,
                split_keys, kN);
  if (num_seqs == 0 || max_q_len == 0 || num_query_rows == 0) return PS_OK;
  if (num_seqs > 65535 || num_kv_heads > 65535 || num_query_rows >= (int64_t(1) << 31))
    return fail(PS_ERR_INVALID, "%s: too many sequences/heads/rows for one launch", fn);
  if (!out || !query || !k_pool || !v_pool || !block_tables || !q_starts || !q_lens || !ctx_lens)
    return fail(PS_ERR_INVALID, "%s: null pointer argument", fn);
  if (block_table_stride < max_blocks_per_seq)
    return fail(PS_ERR_INVALID, "%s: block_table_stride < max_blocks_per_seq", fn);
  if (query_token_stride < static_cast<int64_t>(num_q_heads) * head_dim ||
      out_token_stride < static_cast<int64_t>(num_q_heads) * head_dim ||
      (query_token_stride % 8) || (out_token_stride % 8) || !aligned(query, 16) ||
      !aligned(out, 16) || !aligned(k_pool, 16) || !aligned(v_pool, 16))
    return fail(PS_ERR_INVALID, "%s: tensors must be 16-byte aligned with strides >= Hq*D, %% 8",
                fn);
  const int64_t rows = num_blocks * num_kv_heads * block_size;
  if (rows >= (int64_t(1) << 31))
    return fail(PS_ERR_INVALID, "%s: pool too large for 32-bit TMA row coordinates", fn);

  const int tpt = kM / group;
  PrefillParams p{};
  p.out = out;
  p.out_stride = out_token_stride;
  p.block_tables = block_tables;
  p.bt_stride = block_table_stride;
  p.q_starts = q_starts;
  p.q_lens = q_lens;
  p.ctx_lens = ctx_lens;
  p.num_blocks = num_blocks;
  p.num_rows = num_query_rows;
  p.num_kv_heads = num_kv_heads;
  p.num_q_heads = num_q_heads;
  p.group = group;
  p.tokens_per_tile = tpt;
  p.max_blocks = max_blocks_per_seq;
  p.block_size = block_size;
  p.num_seqs = num_seqs;
  p.num_q_tiles = (max_q_len + 2 * tpt - 1) / (2 * tpt);
  const SplitGeometry sg = split_geometry(num_seqs, max_q_len, group, num_kv_heads, head_dim,
                                          block_size, max_blocks_per_seq, split_keys);
  const int64_t items = sg.items;
  if (sg.units >= (int64_t(1) << 31) || sg.units * 2 * kM / kCombineWarps >= (int64_t(1) << 31))
    return fail(PS_ERR_INVALID, "%s: too many query tiles for one launch", fn);
  p.num_items = static_cast<int>(items);
  p.splits = sg.splits;
  p.split_tiles = sg.split_tiles;
  p.num_units = static_cast<int>(sg.units);
  if (sg.splits > 1) {
    if (!workspace || !aligned(workspace, 256))
      return fail(PS_ERR_INVALID, "%s: split-K needs a 256-byte aligned workspace", fn);
    if (workspace_bytes < sg.workspace_bytes())
      return fail(PS_ERR_INVALID, "%s: workspace of %lld bytes, %lld needed", fn,
                  static_cast<long long>(workspace_bytes),
                  static_cast<long long>(sg.workspace_bytes()));
    p.part_o = static_cast<float*>(workspace);
    p.part_ml = reinterpret_cast<float2*>(static_cast<uint8_t*>(workspace) +
                                          (sg.o_bytes + 255) / 256 * 256);
  }
  p.scale_log2 = scale * 1.4426950408889634f;
  p.err = device_error;

  CUtensorMap qm, km, vm;
  {
    // query viewed as [rows][Hq][D]: box = 64 dims x G heads x tpt tokens.
    const uint64_t dims[3] = {static_cast<uint64_t>(head_dim), static_cast<uint64_t>(num_q_heads),
                              static_cast<uint64_t>(num_query_rows)};
    const uint64_t strides[2] = {static_cast<uint64_t>(head_dim) * 2,
                                 static_cast<uint64_t>(query_token_stride) * 2};
    const uint32_t box[3] = {64, static_cast<uint32_t>(group), static_cast<uint32_t>(tpt)};
    int st = encode_tmap_16bit(&qm, const_cast<void*>(query), 3, dims, strides, box,
                               CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != PS_OK) return st;
  }
  int st = get_pool_tmap(k_pool, static_cast<uint64_t>(rows), head_dim, block_size, &km);
  if (st != PS_OK) return st;
  st = get_pool_tmap(v_pool, static_cast<uint64_t>(rows), head_dim, block_size, &vm);
  if (st != PS_OK) return st;

  cudaStream_t s = as_stream(stream);
  // Persistent: one CTA per SM (shared memory allows no more), at most one per unit.
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  dim3 grid(static_cast<unsigned>(std::min<int64_t>(sg.units, sms)));
  return dispatch_prefill(p, qm, km, vm, grid, s, dtype, head_dim, block_size);
}

}  // namespace
}  // namespace ps

using namespace ps;

extern "C" int ps_paged_prefill(void* out, int64_t out_token_stride, const void* query,
                                int64_t query_token_stride, int64_t num_query_rows,
                                const void* k_pool, const void* v_pool, int64_t num_blocks,
                                const int32_t* block_tables, int64_t block_table_stride,
                                const int32_t* q_starts, const int32_t* q_lens,
                                const int32_t* ctx_lens, int num_seqs, int max_q_len,
                                int num_q_heads, int num_kv_heads, int head_dim, int block_size,
                                int max_blocks_per_seq, float scale, int dtype,
                                int32_t* device_error, void* stream) {
  ps::NvtxRange nvtx_range("ps_paged_prefill");
  return prefill_entry("ps_paged_prefill", out, out_token_stride, query, query_token_stride,
                       num_query_rows, k_pool, v_pool, num_blocks, block_tables,
                       block_table_stride, q_starts, q_lens, ctx_lens, num_seqs, max_q_len,
                       num_q_heads, num_kv_heads, head_dim, block_size, max_blocks_per_seq, scale,
                       0, nullptr, 0, dtype, device_error, stream);
}

extern "C" int ps_paged_prefill_split(void* out, int64_t out_token_stride, const void* query,
                                      int64_t query_token_stride, int64_t num_query_rows,
                                      const void* k_pool, const void* v_pool, int64_t num_blocks,
                                      const int32_t* block_tables, int64_t block_table_stride,
                                      const int32_t* q_starts, const int32_t* q_lens,
                                      const int32_t* ctx_lens, int num_seqs, int max_q_len,
                                      int num_q_heads, int num_kv_heads, int head_dim,
                                      int block_size, int max_blocks_per_seq, float scale,
                                      int split_keys, void* workspace, int64_t workspace_bytes,
                                      int dtype, int32_t* device_error, void* stream) {
  ps::NvtxRange nvtx_range("ps_paged_prefill_split");
  return prefill_entry("ps_paged_prefill_split", out, out_token_stride, query,
                       query_token_stride, num_query_rows, k_pool, v_pool, num_blocks,
                       block_tables, block_table_stride, q_starts, q_lens, ctx_lens, num_seqs,
                       max_q_len, num_q_heads, num_kv_heads, head_dim, block_size,
                       max_blocks_per_seq, scale, split_keys, workspace, workspace_bytes, dtype,
                       device_error, stream);
}

extern "C" int64_t ps_paged_prefill_workspace_bytes(int num_seqs, int max_q_len,
                                                    int num_q_heads, int num_kv_heads,
                                                    int head_dim, int block_size,
                                                    int max_blocks_per_seq, int split_keys) {
  if (num_seqs <= 0 || max_q_len <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 ||
      num_q_heads % num_kv_heads || num_q_heads / num_kv_heads > 16 ||
      (head_dim != 64 && head_dim != 128) || block_size <= 0 || max_blocks_per_seq <= 0 ||
      split_keys < 0 || split_keys % kN)
    return 0;
  return split_geometry(num_seqs, max_q_len, num_q_heads / num_kv_heads, num_kv_heads, head_dim,
                        block_size, max_blocks_per_seq, split_keys)
      .workspace_bytes();
}
