// Causal paged prefill on tcgen05 tensor cores (sm_100a).
//
// One CTA (one per SM) owns two 128-row query tiles A and B of the same
// (sequence, KV head): tile A = tokens [t0, t0+tpt), tile B = the next tpt
// tokens; a row = (token, one of the G = Hq/Hkv query heads of the group), so
// every K/V tile loaded feeds 2 x 128 query rows. Keys stream in tiles of 64
// (four 16-token blocks found through the block table) through a 5-stage
// shared-memory ring that both query tiles read.
//
//   warp 8 (TMA)    : Q_A, Q_B once (3-D boxes: 64 dims x G heads x tpt tokens,
//                     128B swizzle); then K_j, V_j per key tile (64-column boxes).
//   warp 9 (MMA)    : one elected thread issues tcgen05.mma (kind::f16, fp32
//                     accumulators in TMEM):
//                       S_X(j) = Q_X K_j^T  (M128 N64, 8 x K16; A, B K-major in smem)
//                       O_X   += P_X(j) V_j (M128 N128, 4 x K16; A = P_X in TMEM,
//                                            B = V_j MN-major in smem)
//                     S of both tiles for key tile j+1 is issued before P(j) is
//                     awaited, so the tensor core computes it while the
//                     softmax warps work on tile j.
//   warps 0-3 / 4-7 : softmax of tile A / B; thread = TMEM lane = row:
//                     tcgen05.ld of S_X(j), causal mask on diagonal key tiles only,
//                     online softmax in the log2 domain (scale folded into one
//                     packed FFMA, ex2.approx), P_X(j) (bf16/f16) written with
//                     tcgen05.st over the first 32 columns of the S buffer it came
//                     from, O_X rescaled in TMEM only when a row max grows by > 2^8
//                     (the only step that waits for a PV), O_X / l stored at the end.
//
// TMEM: S_A / S_B double-buffered (4 x 64 cols, P aliased), O_A, O_B (2 x 128) = 512.
// S_X(j+2) overwrites P_X(j) only after PV_X(j) was issued by the same thread.
// Barrier phases: a waiter must never fall two completions behind, or its parity
// wait aliases. The softmax of a tile can finish key tiles j and j+1 before the
// MMA thread looks for P(j) (S(j+1) is issued first), so the P barriers, like
// the S and O ones, are kept per S buffer: each completes once per two tiles.
// All waits are bounded; a timeout sets PS_DEVERR_TIMEOUT and a shared abort
// flag so every role leaves its loop, drains its in-flight copies / MMAs and
// frees TMEM before the CTA exits.
#include <type_traits>

#include "capi_internal.h"
#include "common.cuh"
#include "tcgen05.cuh"

namespace ps {
namespace {

constexpr int kBS = 16;   // tokens per KV block
constexpr int kM = 128;   // query rows per query tile
constexpr int kN = 64;    // keys per KV tile
constexpr int kD = 128;   // head dim
constexpr int kTileBlocks = kN / kBS;
constexpr int kQHalf = kM * 128;           // one 64-column half of a Q tile: [128 rows][128 B]
constexpr int kQBytes = 2 * kQHalf;        // 32 KB per query tile
constexpr int kKVHalf = kN * 128;          // [64 keys][128 B]
constexpr int kKVBytes = 2 * kKVHalf;      // 16 KB (K or V of one key tile)
constexpr int kStageBytes = 2 * kKVBytes;  // K + V
constexpr int kStages = 5;
constexpr int kOffQ = 0;                   // Q_A, Q_B
constexpr int kOffStage = 2 * kQBytes;
constexpr int kOffBars = kOffStage + kStages * kStageBytes;
enum : int {
  kBarQ = 0,
  kBarKVFull = 1,                      // [kStages]
  kBarKVEmpty = kBarKVFull + kStages,  // [kStages]
  kBarSFull = kBarKVEmpty + kStages,   // [tile][S buffer]
  kBarP = kBarSFull + 4,               // [tile][S buffer]: P_X(j) written (128 arrivals)
  kBarOBuf = kBarP + 4,                // [tile][S buffer of the P it consumed]
  kBarOFinal = kBarOBuf + 4,           // [tile]: the last PV of the tile
  kBarDone = kBarOFinal + 2,
  kNumBars = kBarDone + 1
};
constexpr int kOffMisc = kOffBars + kNumBars * 8;  // [0] TMEM base, [1] abort flag
constexpr size_t kSmemBytes = 1024 + kOffMisc + 16;
static_assert(kSmemBytes <= 232448, "exceeds the per-block shared memory limit");
constexpr int kThreads = 320;
constexpr int kWarpTma = 8;
constexpr int kWarpMma = 9;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemS = 0;    // S_X buffer k (P_X in its first 32 columns) at (2X + k) * 64
constexpr uint32_t kTmemO = 256;  // O_X at kTmemO + X * 128
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
  float scale_log2;
  int32_t* err;
};

// Bounded mbarrier wait that also gives up when another role aborted.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort,
                                              int32_t* err) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 1023u) == 1023u && *abort) return false;
  }
  *abort = 1;
  set_device_error(err, PS_DEVERR_TIMEOUT);
  return false;
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
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
template <typename T>
__device__ __forceinline__ void softmax_tile(const PrefillParams& p, uint64_t* bars,
                                             volatile int* abort, uint32_t tmem, int tile, int r,
                                             int warp_in_tile, int ntiles, int t0_tile, int ctx,
                                             int q_len, int q_start, int h, int last_key) {
  const int G = p.group;
  const int tpt = p.tokens_per_tile;
  const int tok = r / G;
  const bool row_real = (r < G * tpt) && (t0_tile + tok < q_len);
  const int limit = row_real ? ctx + t0_tile + tok : last_key - 1;  // last key this row sees
  const int tile_min_limit = ctx + t0_tile;  // smallest limit among this tile's real rows
  const uint32_t lane_tmem = tmem + (static_cast<uint32_t>(warp_in_tile * 32) << 16);
  const uint32_t o_col = kTmemO + tile * kD;
  const float2 scale2 = make_float2(p.scale_log2, p.scale_log2);
  float m_used = -INFINITY;  // running max, log2-scaled
  float l_sum = 0.f;
  bool ok = true;
  for (int j = 0; j < ntiles; ++j) {
    const int buf = j & 1;
    const uint32_t s_col = kTmemS + (2 * tile + buf) * kN;
    ok = wait_or_abort(&bars[kBarSFull + 2 * tile + buf], (j >> 1) & 1, abort, p.err);
    ok = __all_sync(0xffffffffu, ok);
    if (!ok) break;
    tc_fence_after();
    uint32_t sraw[2][32];
    tmem_ld32(lane_tmem + s_col, sraw[0]);
    tmem_ld32(lane_tmem + s_col + 32, sraw[1]);
    tmem_wait_ld();
    float* s = reinterpret_cast<float*>(&sraw[0][0]);
    const int key0 = j * kN;
    if (key0 + kN - 1 > tile_min_limit) {  // diagonal tile: causal mask (warp-uniform test)
#pragma unroll
      for (int c = 0; c < kN; ++c)
        if (key0 + c > limit) s[c] = -INFINITY;
    }
    float mx[4] = {s[0], s[1], s[2], s[3]};
#pragma unroll
    for (int c = 4; c < kN; c += 4) {
      mx[0] = fmaxf(mx[0], s[c]);
      mx[1] = fmaxf(mx[1], s[c + 1]);
      mx[2] = fmaxf(mx[2], s[c + 2]);
      mx[3] = fmaxf(mx[3], s[c + 3]);
    }
    const float mt = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * p.scale_log2;
    const bool rescale = __any_sync(0xffffffffu, mt > m_used + kRescaleThreshold);
    if (rescale) {
      const float m_new = fmaxf(m_used, mt);
      const float alpha = (m_new == -INFINITY) ? 1.f : ex2_approx(m_used - m_new);
      if (j > 0) {
        // O_X must hold every PV up to j-1 before it is rescaled.
        const int pb = (j - 1) & 1;
        ok = wait_or_abort(&bars[kBarOBuf + 2 * tile + pb], ((j - 1) >> 1) & 1, abort, p.err);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        const float2 a2 = make_float2(alpha, alpha);
#pragma unroll
        for (int c = 0; c < kD / 32; ++c) {
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
      l_sum *= alpha;
      m_used = m_new;
    }
    // p = 2^(s*scale - m) -> P_X(j) as packed pairs (lane r = row r) over the
    // first 32 columns of this S buffer; the row sum uses the rounded P.
    const float2 negm = make_float2(-m_used, -m_used);
    float2 ls = make_float2(0.f, 0.f);
    uint32_t packed[kN / 2];
#pragma unroll
    for (int c = 0; c < kN; c += 2) {
      const float2 x = __ffma2_rn(make_float2(s[c], s[c + 1]), scale2, negm);
      packed[c >> 1] = pack2<T>(ex2_approx(x.x), ex2_approx(x.y));
      ls = __fadd2_rn(ls, unpack2<T>(packed[c >> 1]));
    }
    l_sum += ls.x + ls.y;
    tmem_st32(lane_tmem + s_col, packed);
    tmem_wait_st();
    tc_fence_before();
    mbar_arrive(&bars[kBarP + 2 * tile + buf]);
  }
  if (ok) {
    ok = wait_or_abort(&bars[kBarOFinal + tile], 0, abort, p.err);
    ok = __all_sync(0xffffffffu, ok);
  }
  if (!ok) return;
  tc_fence_after();
  const float inv = (l_sum > 0.f) ? 1.f / l_sum : 0.f;
  const int64_t out_row = static_cast<int64_t>(q_start) + t0_tile + tok;
  T* orow = static_cast<T*>(p.out) + out_row * p.out_stride +
            static_cast<int64_t>(h * G + (r % G)) * kD;
#pragma unroll
  for (int c = 0; c < kD / 32; ++c) {
    uint32_t o[32];
    tmem_ld32(lane_tmem + o_col + c * 32, o);
    tmem_wait_ld();
    if (row_real) {
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        uint4 w;
        w.x = pack2<T>(__uint_as_float(o[8 * v + 0]) * inv, __uint_as_float(o[8 * v + 1]) * inv);
        w.y = pack2<T>(__uint_as_float(o[8 * v + 2]) * inv, __uint_as_float(o[8 * v + 3]) * inv);
        w.z = pack2<T>(__uint_as_float(o[8 * v + 4]) * inv, __uint_as_float(o[8 * v + 5]) * inv);
        w.w = pack2<T>(__uint_as_float(o[8 * v + 6]) * inv, __uint_as_float(o[8 * v + 7]) * inv);
        *reinterpret_cast<uint4*>(orow + c * 32 + 8 * v) = w;
      }
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    paged_prefill_kernel(const PrefillParams p, const __grid_constant__ CUtensorMap qmap,
                         const __grid_constant__ CUtensorMap kmap,
                         const __grid_constant__ CUtensorMap vmap) {
  const int qt = blockIdx.x;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int q_len = p.q_lens[b];
  const int tpt = p.tokens_per_tile;
  const int t0 = qt * 2 * tpt;
  if (t0 >= q_len) return;  // uniform: nothing allocated yet
  const int ctx = p.ctx_lens[b];
  const int q_start = p.q_starts[b];
  const int total = ctx + q_len;
  if (ctx < 0 || q_start < 0 || static_cast<int64_t>(q_start) + q_len > p.num_rows ||
      total > p.max_blocks * kBS) {
    if (threadIdx.x == 0) set_device_error(p.err, PS_DEVERR_LENGTH);
    return;
  }
  const int G = p.group;
  const int rows_here = min(2 * tpt, q_len - t0);
  const int last_key = ctx + t0 + rows_here;  // keys [0, last_key) are needed
  const int ntiles = (last_key + kN - 1) / kN;
  const int nblk_seq = (total + kBS - 1) / kBS;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBars);
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  volatile int* abort = reinterpret_cast<volatile int*>(misc + 1);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumBars; ++i) mbar_init(&bars[i], (i >= kBarP && i < kBarP + 4) ? 128 : 1);
    *abort = 0;
    fence_barrier_init();
  }
  if (warp == kWarpMma) tmem_alloc(&misc[0], kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = misc[0];
  const int32_t* bt = p.block_tables + static_cast<int64_t>(b) * p.bt_stride;

  if (warp == kWarpTma) {
    // ------------------------------------------------------------ TMA producer
    // The whole warp walks the tiles so block ids arrive 32 at a time (one
    // coalesced load per 8 key tiles, shuffled to lane 0) instead of one L2
    // round trip per block; lane 0 issues every barrier op and TMA load.
    if (lane == 0) {
      tma_prefetch_desc(&qmap);
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
      mbar_arrive_expect_tx(&bars[kBarQ], 2u * 2u * 64u * G * tpt * 2u);
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        uint8_t* q = smem + kOffQ + x * kQBytes;
        tma_load_3d(q, &qmap, &bars[kBarQ], 0, h * G, q_start + t0 + x * tpt);
        tma_load_3d(q + kQHalf, &qmap, &bars[kBarQ], 64, h * G, q_start + t0 + x * tpt);
      }
    }
    int issued = 0;
    int window = -32;  // first block index held by the lanes' `my_row`
    int32_t my_row = 0;
    for (int j = 0; j < ntiles; ++j) {
      const int kb0 = j * kTileBlocks;
      if (kb0 >= window + 32) {
        window = kb0;
        const int kb = window + lane;
        int32_t id = 0;
        if (kb < nblk_seq) {
          id = bt[kb];
          if (id < 0 || id >= p.num_blocks) {
            set_device_error(p.err, PS_DEVERR_BLOCK_ID);
            id = 0;
          }
        }
        my_row = kb < nblk_seq ? (id * p.num_kv_heads + h) * kBS : -1;
      }
      int32_t rows[kTileBlocks];
#pragma unroll
      for (int bb = 0; bb < kTileBlocks; ++bb) rows[bb] = __shfl_sync(0xffffffffu, my_row, kb0 - window + bb);
#pragma unroll
      for (int bb = 1; bb < kTileBlocks; ++bb)  // past the sequence end: re-read a valid block (masked)
        if (rows[bb] < 0) rows[bb] = rows[0];
      bool ok = true;
      if (lane == 0) {
        const int st = j % kStages;
        if (j >= kStages)
          ok = wait_or_abort(&bars[kBarKVEmpty + st], ((j / kStages) - 1) & 1, abort, p.err);
        if (ok) {
          uint8_t* kdst = smem + kOffStage + st * kStageBytes;
          uint8_t* vdst = kdst + kKVBytes;
          mbar_arrive_expect_tx(&bars[kBarKVFull + st], kStageBytes);
#pragma unroll
          for (int bb = 0; bb < kTileBlocks; ++bb) {
            tma_load_2d(kdst + bb * (kBS * 128), &kmap, &bars[kBarKVFull + st], 0, rows[bb]);
            tma_load_2d(kdst + kKVHalf + bb * (kBS * 128), &kmap, &bars[kBarKVFull + st], 64,
                        rows[bb]);
            tma_load_2d(vdst + bb * (kBS * 128), &vmap, &bars[kBarKVFull + st], 0, rows[bb]);
            tma_load_2d(vdst + kKVHalf + bb * (kBS * 128), &vmap, &bars[kBarKVFull + st], 64,
                        rows[bb]);
          }
        }
      }
      if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
      issued = j + 1;
    }
    if (lane == 0) {
      // Drain: the Q tiles and the last load issued into each stage have landed.
      (void)mbar_wait_bounded(&bars[kBarQ], 0);
      for (int j = max(0, issued - kStages); j < issued; ++j)
        (void)mbar_wait_bounded(&bars[kBarKVFull + (j % kStages)], (j / kStages) & 1);
    }
  } else if (warp == kWarpMma) {
    // ------------------------------------------------------------ MMA issuer
    // The whole warp runs this loop (waits, descriptor arithmetic: all
    // warp-uniform); one elected lane issues each tcgen05.mma / commit.
    const bool leader = elect_one();
    constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
    constexpr uint32_t kIdS = idesc_f16(kBf16, kM, kN, false, false);
    constexpr uint32_t kIdO = idesc_f16(kBf16, kM, kD, false, true);
    // Descriptors are built once; stepping through K, stages and buffers only
    // adds (byte offset >> 4) to the start-address field (addresses < 256 KB,
    // so the 14-bit field never carries).
    const uint64_t q_desc = sdesc_sw128(smem_u32(smem + kOffQ), 16, 1024);
    const uint64_t k_desc = sdesc_sw128(smem_u32(smem + kOffStage), 16, 1024);
    const uint64_t v_desc = sdesc_sw128(smem_u32(smem + kOffStage + kKVBytes), kKVHalf, 1024);
    auto wait_all = [&](uint64_t* bar, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, wait_or_abort(bar, parity, abort, p.err));
    };
    // S_X(j) into S buffer j&1 of tile X (K_j's stage must be full).
    auto issue_s = [&](int x, int j) {
      const uint64_t kd = k_desc + static_cast<uint64_t>(((j % kStages) * kStageBytes) >> 4);
      const uint32_t d = tmem + kTmemS + (2 * x + (j & 1)) * kN;
      const uint64_t qd = q_desc + static_cast<uint64_t>(x * (kQBytes >> 4));
#pragma unroll
      for (int kk = 0; kk < kD / 16; ++kk) {
        const uint32_t off = ((kk >> 2) * kQHalf + (kk & 3) * 32) >> 4;
        const uint32_t koff = ((kk >> 2) * kKVHalf + (kk & 3) * 32) >> 4;
        if (leader) umma_f16(d, qd + off, kd + koff, kIdS, kk > 0 ? 1u : 0u);
      }
      if (leader) umma_commit(&bars[kBarSFull + 2 * x + (j & 1)]);
    };
    // O_X += P_X(j) V_j once the softmax of tile X has written P_X(j).
    auto issue_pv = [&](int x, int j) -> bool {
      if (!wait_all(&bars[kBarP + 2 * x + (j & 1)], (j >> 1) & 1)) return false;
      tc_fence_after();
      const uint64_t vd = v_desc + static_cast<uint64_t>(((j % kStages) * kStageBytes) >> 4);
      const uint32_t p_tmem = tmem + kTmemS + (2 * x + (j & 1)) * kN;
#pragma unroll
      for (int kk = 0; kk < kN / 16; ++kk) {
        if (leader)
          umma_f16_ts(tmem + kTmemO + x * kD, p_tmem + kk * 8, vd + (kk * 2048 >> 4), kIdO,
                      (j > 0 || kk > 0) ? 1u : 0u);
      }
      if (leader) {
        umma_commit(&bars[kBarOBuf + 2 * x + (j & 1)]);
        if (j + 1 == ntiles) umma_commit(&bars[kBarOFinal + x]);
      }
      return true;
    };
    // Issue order per key tile j: S_A(j+1), PV_A(j), S_B(j+1), PV_B(j). Each
    // wait sits behind a batch of queued MMAs, so the tensor pipe stays fed
    // while the warp polls; S of the next tile overlaps the softmax of this one.
    bool ok = wait_all(&bars[kBarQ], 0) && wait_all(&bars[kBarKVFull], 0);
    if (ok) {
      tc_fence_after();
      issue_s(0, 0);
      issue_s(1, 0);
    }
    for (int j = 0; ok && j < ntiles; ++j) {
      const bool more = j + 1 < ntiles;
      if (more) {
        ok = wait_all(&bars[kBarKVFull + (j + 1) % kStages], ((j + 1) / kStages) & 1);
        if (!ok) break;
        tc_fence_after();
        issue_s(0, j + 1);
      }
      if (!(ok = issue_pv(0, j))) break;
      if (more) issue_s(1, j + 1);
      if (!(ok = issue_pv(1, j))) break;
      if (leader) umma_commit(&bars[kBarKVEmpty + j % kStages]);
    }
    // Every MMA issued above has completed before TMEM is released.
    if (leader) umma_commit(&bars[kBarDone]);
    __syncwarp();
    (void)mbar_wait_bounded(&bars[kBarDone], 0);
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int x = warp >> 2;  // query tile 0 (A) or 1 (B)
    softmax_tile<T>(p, bars, abort, tmem, x, threadIdx.x & 127, warp & 3, ntiles, t0 + x * tpt,
                    ctx, q_len, q_start, h, last_key);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// One per element type: the dynamic shared-memory opt-in is per kernel and per device.
template <typename T>
int launch_prefill(const PrefillParams& p, const CUtensorMap& qm, const CUtensorMap& km,
                   const CUtensorMap& vm, dim3 grid, cudaStream_t s) {
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(paged_prefill_kernel<T>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kSmemBytes));
    if (e != cudaSuccess)
      return fail(PS_ERR_CUDA, "ps_paged_prefill: cannot reserve %zu B shared memory: %s",
                  kSmemBytes, cudaGetErrorString(e));
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  paged_prefill_kernel<T><<<grid, kThreads, kSmemBytes, s>>>(p, qm, km, vm);
  return check_launch("ps_paged_prefill");
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
  const char* fn = "ps_paged_prefill";
  if (dtype != PS_DTYPE_BF16 && dtype != PS_DTYPE_F16)
    return fail(PS_ERR_UNSUPPORTED, "%s: dtype %d unsupported (bf16/f16 only)", fn, dtype);
  if (head_dim != kD)
    return fail(PS_ERR_UNSUPPORTED, "%s: head_dim %d unsupported (128)", fn, head_dim);
  if (block_size != kBS)
    return fail(PS_ERR_UNSUPPORTED, "%s: block_size %d unsupported (16)", fn, block_size);
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
  const int64_t rows = num_blocks * num_kv_heads * kBS;
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
  int st = get_pool_tmap(k_pool, static_cast<uint64_t>(rows), head_dim, kBS, &km);
  if (st != PS_OK) return st;
  st = get_pool_tmap(v_pool, static_cast<uint64_t>(rows), head_dim, kBS, &vm);
  if (st != PS_OK) return st;

  cudaStream_t s = as_stream(stream);
  dim3 grid((max_q_len + 2 * tpt - 1) / (2 * tpt), num_kv_heads, num_seqs);
  if (dtype == PS_DTYPE_BF16) return launch_prefill<__nv_bfloat16>(p, qm, km, vm, grid, s);
  return launch_prefill<__half>(p, qm, km, vm, grid, s);
}
