// Causal paged prefill on tcgen05 tensor cores (sm_100a).
//
// One CTA (one per SM) owns two 128-row query tiles A and B of the same
// (sequence, KV head): tile A = tokens [t0, t0+tpt), tile B = the next tpt
// tokens, each row = (token, one of the G = Hq/Hkv query heads of the group),
// so every K/V tile loaded feeds 2 x 128 query rows. Keys stream in tiles of 64
// (four 16-token blocks found through the block table) through a 4-stage
// shared-memory ring that both query tiles read:
//
//   warp 8 (TMA)       : Q_A, Q_B once (3-D boxes: 64 dims x G heads x tpt
//                        tokens, 128B swizzle); then K_j, V_j per key tile.
//   warp 9 (MMA)       : one elected thread issues tcgen05.mma (kind::f16,
//                        fp32 accumulators in TMEM): S_X(j) = Q_X K_j^T
//                        (M128 N64, 8 x K16, K-major A/B) into a double-buffered
//                        S_X, and O_X += P_X(j) V_j (M128 N128, 4 x K16, K-major
//                        A, MN-major B). S for tile j+1 of both query tiles is
//                        issued before P(j) is awaited, so the tensor core works
//                        on one tile while the softmax warps work on the other.
//   warps 0-3 / 4-7    : softmax of tile A / B; thread = TMEM lane = row:
//                        tcgen05.ld of S, causal mask on diagonal key tiles only,
//                        online softmax in the log2 domain (scale folded into one
//                        packed FFMA, ex2.approx), P (bf16/f16) to shared memory,
//                        O rescaled in TMEM only when a row max grows by > 2^8,
//                        O / l stored to global at the end.
//
// TMEM: S_A (2 x 64 cols), S_B (2 x 64), O_A (128), O_B (128) = 512 columns.
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
constexpr int kPBytes = kM * kN * 2;       // 16 KB: P of one query tile, [128 rows][128 B]
constexpr int kKVHalf = kN * 128;          // [64 rows][128 B]
constexpr int kKVBytes = 2 * kKVHalf;      // 16 KB (K or V of one key tile)
constexpr int kStageBytes = 2 * kKVBytes;  // K + V
constexpr int kStages = 4;
constexpr int kOffQ = 0;                   // Q_A, Q_B
constexpr int kOffP = 2 * kQBytes;         // P_A, P_B
constexpr int kOffStage = kOffP + 2 * kPBytes;
constexpr int kOffBars = kOffStage + kStages * kStageBytes;
enum : int {
  kBarQ = 0,
  kBarKVFull = 1,                      // [kStages]
  kBarKVEmpty = kBarKVFull + kStages,  // [kStages]
  kBarSFull = kBarKVEmpty + kStages,   // [tile][2 buffers]
  kBarP = kBarSFull + 4,               // [tile]
  kBarO = kBarP + 2,                   // [tile]
  kBarDone = kBarO + 2,
  kNumBars = kBarDone + 1
};
constexpr int kOffMisc = kOffBars + kNumBars * 8;  // [0] TMEM base, [1] abort flag
constexpr size_t kSmemBytes = 1024 + kOffMisc + 16;
static_assert(kSmemBytes <= 232448, "exceeds the per-block shared memory limit");
constexpr int kThreads = 320;
constexpr int kWarpTma = 8;
constexpr int kWarpMma = 9;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemS = 0;    // S_X buffer k at kTmemS + (2X + k) * 64
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

// Softmax + epilogue of one query tile; 128 threads, thread = TMEM lane = row.
template <typename T>
__device__ __forceinline__ void softmax_tile(const PrefillParams& p, uint8_t* smem,
                                             uint64_t* bars, volatile int* abort, uint32_t tmem,
                                             int tile, int r, int warp_in_tile, int ntiles,
                                             int t0_tile, int ctx, int q_len, int q_start, int h,
                                             int last_key) {
  const int G = p.group;
  const int tpt = p.tokens_per_tile;
  const int tok = r / G;
  const bool row_real = (r < G * tpt) && (t0_tile + tok < q_len);
  const int limit = row_real ? ctx + t0_tile + tok : last_key - 1;  // last key this row sees
  const int tile_min_limit = ctx + t0_tile;  // smallest limit among this tile's real rows
  const uint32_t lane_tmem = tmem + (static_cast<uint32_t>(warp_in_tile * 32) << 16);
  const uint32_t s_col = kTmemS + tile * 2 * kN;
  const uint32_t o_col = kTmemO + tile * kD;
  uint64_t* bar_s = &bars[kBarSFull + tile * 2];
  uint64_t* bar_p = &bars[kBarP + tile];
  uint64_t* bar_o = &bars[kBarO + tile];
  uint8_t* prow = smem + kOffP + tile * kPBytes + r * 128;
  const float2 scale2 = make_float2(p.scale_log2, p.scale_log2);
  float m_used = -INFINITY;  // running max, log2-scaled
  float l_sum = 0.f;
  bool ok = true;
  for (int j = 0; j < ntiles; ++j) {
    ok = wait_or_abort(&bar_s[j & 1], (j >> 1) & 1, abort, p.err);
    ok = __all_sync(0xffffffffu, ok);
    if (!ok) break;
    tc_fence_after();
    uint32_t sraw[2][32];
    tmem_ld32(lane_tmem + s_col + (j & 1) * kN, sraw[0]);
    tmem_ld32(lane_tmem + s_col + (j & 1) * kN + 32, sraw[1]);
    tmem_wait_ld();
    float* s = reinterpret_cast<float*>(&sraw[0][0]);
    const int key0 = j * kN;
    if (key0 + kN - 1 > tile_min_limit) {  // diagonal tile: causal mask (warp-uniform test)
#pragma unroll
      for (int c = 0; c < kN; ++c)
        if (key0 + c > limit) s[c] = -INFINITY;
    }
    float mraw = s[0];
#pragma unroll
    for (int c = 1; c < kN; ++c) mraw = fmaxf(mraw, s[c]);
    const float mt = mraw * p.scale_log2;  // max of the scaled scores (scale > 0)
    if (j > 0) {
      // PV_X(j-1) finished: O_X is stable and P_X may be overwritten.
      ok = wait_or_abort(bar_o, (j - 1) & 1, abort, p.err);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
    }
    const bool need = mt > m_used + kRescaleThreshold;
    if (__any_sync(0xffffffffu, need)) {
      const float m_new = fmaxf(m_used, mt);
      const float alpha = (m_new == -INFINITY) ? 1.f : ex2_approx(m_used - m_new);
      if (j > 0) {
        const float2 a2 = make_float2(alpha, alpha);
#pragma unroll
        for (int c = 0; c < kD / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(lane_tmem + o_col + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            const float2 v = __fmul2_rn(make_float2(__uint_as_float(o[e]), __uint_as_float(o[e + 1])), a2);
            o[e] = __float_as_uint(v.x);
            o[e + 1] = __float_as_uint(v.y);
          }
          tmem_st32(lane_tmem + o_col + c * 32, o);
        }
        tmem_wait_st();
      }
      l_sum *= alpha;
      m_used = m_new;
    }
    // p = 2^(s*scale - m); the row sum uses the rounded P the MMA multiplies with.
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
#pragma unroll
    for (int c8 = 0; c8 < 8; ++c8) {
      *reinterpret_cast<uint4*>(prow + ((c8 ^ (r & 7)) << 4)) =
          make_uint4(packed[4 * c8], packed[4 * c8 + 1], packed[4 * c8 + 2], packed[4 * c8 + 3]);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    mbar_arrive(bar_p);
  }
  if (ok) {
    ok = wait_or_abort(bar_o, (ntiles - 1) & 1, abort, p.err);
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
    mbar_init(&bars[kBarQ], 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars[kBarKVFull + s], 1);
      mbar_init(&bars[kBarKVEmpty + s], 1);
    }
    for (int i = 0; i < 4; ++i) mbar_init(&bars[kBarSFull + i], 1);
    for (int x = 0; x < 2; ++x) {
      mbar_init(&bars[kBarP + x], 128);
      mbar_init(&bars[kBarO + x], 1);
    }
    mbar_init(&bars[kBarDone], 1);
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
      int issued = 0;
      for (int j = 0; j < ntiles; ++j) {
        const int st = j % kStages;
        if (j >= kStages &&
            !wait_or_abort(&bars[kBarKVEmpty + st], ((j / kStages) - 1) & 1, abort, p.err))
          break;
        uint8_t* kdst = smem + kOffStage + st * kStageBytes;
        uint8_t* vdst = kdst + kKVBytes;
        mbar_arrive_expect_tx(&bars[kBarKVFull + st], kStageBytes);
        int32_t first = bt[j * kTileBlocks];
        if (first < 0 || first >= p.num_blocks) {
          set_device_error(p.err, PS_DEVERR_BLOCK_ID);
          first = 0;
        }
#pragma unroll
        for (int bb = 0; bb < kTileBlocks; ++bb) {
          const int kb = j * kTileBlocks + bb;
          int32_t id = first;  // blocks past the sequence end re-read a valid block (masked)
          if (bb > 0 && kb < nblk_seq) {
            id = bt[kb];
            if (id < 0 || id >= p.num_blocks) {
              set_device_error(p.err, PS_DEVERR_BLOCK_ID);
              id = 0;
            }
          }
          const int32_t row = (id * p.num_kv_heads + h) * kBS;
          tma_load_2d(kdst + bb * (kBS * 128), &kmap, &bars[kBarKVFull + st], 0, row);
          tma_load_2d(kdst + kKVHalf + bb * (kBS * 128), &kmap, &bars[kBarKVFull + st], 64, row);
          tma_load_2d(vdst + bb * (kBS * 128), &vmap, &bars[kBarKVFull + st], 0, row);
          tma_load_2d(vdst + kKVHalf + bb * (kBS * 128), &vmap, &bars[kBarKVFull + st], 64, row);
        }
        issued = j + 1;
      }
      // Drain: the Q tiles and the last load issued into each stage have landed.
      (void)mbar_wait_bounded(&bars[kBarQ], 0);
      for (int j = max(0, issued - kStages); j < issued; ++j)
        (void)mbar_wait_bounded(&bars[kBarKVFull + (j % kStages)], (j / kStages) & 1);
    }
  } else if (warp == kWarpMma) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
      constexpr uint32_t kIdS = idesc_f16(kBf16, kM, kN, false, false);
      constexpr uint32_t kIdO = idesc_f16(kBf16, kM, kD, false, true);
      const uint32_t q_base = smem_u32(smem + kOffQ);
      const uint32_t p_base = smem_u32(smem + kOffP);
      bool ok = wait_or_abort(&bars[kBarQ], 0, abort, p.err);
      tc_fence_after();
      // S_A(j), S_B(j) into buffer j&1 of each tile.
      auto issue_s = [&](int j) -> bool {
        const int st = j % kStages;
        if (!wait_or_abort(&bars[kBarKVFull + st], (j / kStages) & 1, abort, p.err)) return false;
        tc_fence_after();
        const uint32_t k_base = smem_u32(smem + kOffStage + st * kStageBytes);
#pragma unroll
        for (int x = 0; x < 2; ++x) {
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk) {
            const uint32_t off = (kk >> 2) * kQHalf + (kk & 3) * 32;
            const uint64_t a = sdesc_sw128(q_base + x * kQBytes + off, 16, 1024);
            const uint64_t bd =
                sdesc_sw128(k_base + (kk >> 2) * kKVHalf + (kk & 3) * 32, 16, 1024);
            umma_f16(tmem + kTmemS + (2 * x + (j & 1)) * kN, a, bd, kIdS, kk > 0 ? 1u : 0u);
          }
          umma_commit(&bars[kBarSFull + 2 * x + (j & 1)]);
        }
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; ok && j < ntiles; ++j) {
        if (j + 1 < ntiles && !issue_s(j + 1)) break;
        const int st = j % kStages;
        const uint32_t v_base = smem_u32(smem + kOffStage + st * kStageBytes + kKVBytes);
        bool good = true;
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          if (!wait_or_abort(&bars[kBarP + x], j & 1, abort, p.err)) {
            good = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < kN / 16; ++kk) {
            const uint64_t a = sdesc_sw128(p_base + x * kPBytes + kk * 32, 16, 1024);
            const uint64_t bd = sdesc_sw128(v_base + kk * 2048, kKVHalf, 1024);
            umma_f16(tmem + kTmemO + x * kD, a, bd, kIdO, (j > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&bars[kBarO + x]);
        }
        if (!good) break;
        umma_commit(&bars[kBarKVEmpty + st]);
      }
      // Every MMA issued above has completed before TMEM is released.
      umma_commit(&bars[kBarDone]);
      (void)mbar_wait_bounded(&bars[kBarDone], 0);
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int x = warp >> 2;  // query tile 0 (A) or 1 (B)
    softmax_tile<T>(p, smem, bars, abort, tmem, x, threadIdx.x & 127, warp & 3, ntiles,
                    t0 + x * tpt, ctx, q_len, q_start, h, last_key);
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
