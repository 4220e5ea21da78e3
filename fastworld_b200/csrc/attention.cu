// Flash-style attention forward on tcgen05 for sm_100a (non-causal, head_dim 128).
//
// Replaces flash_attn_varlen_func in the reference forward (fastworld/models/mg2/static.py:
// 138-143): self-attention over [history | current] keys (static.py:213-216) and cross-attention
// over the 257 image-context tokens (static.py:187-192).  Keys come in two segments (the
// per-layer history buffer, then the current chunk) whose lengths are read from device memory,
// so one captured graph serves chunk 0 (no history) and steady chunks, with no host cu_seqlens
// and no concatenation.
//
// One CTA per (128-query tile, head); 192 threads:
//   warps 0-3  softmax: thread = query row.  Loads its S row from TMEM, online softmax in the
//              exp2 domain, rescales its O row in TMEM when the running max grows, writes P
//              (bf16) into a 128-byte-swizzled K-major smem tile, final O / l and store.
//   warp 4     TMA producer: Q once; K and V blocks of 128 keys, double-buffered.
//   warp 5     MMA issuer: S_j = Q K_j^T (SS, N = 128) into one of two TMEM S buffers, and
//              O += P_{j-1} V_{j-1} (A = P from smem K-major, B = V from smem MN-major).
// TMEM: S0 cols [0,128), S1 [128,256), O [256,384) of a 512-column allocation.
#include "../../include/fastworld_b200.h"
#include "fw_internal.h"
#include "fw_ptx.cuh"

namespace fw {

namespace attn {
constexpr int BQ = 128, BKV = 128, HD = 128;
constexpr int TILE = 128 * 64 * 2;          // one [128 rows x 64 cols] bf16 swizzled sub-tile
constexpr int Q_OFF = 0;                    // 2 sub-tiles
constexpr int K_OFF = Q_OFF + 2 * TILE;     // 2 stages x 2 sub-tiles
constexpr int V_OFF = K_OFF + 4 * TILE;     // 2 stages x 2 sub-tiles
constexpr int P_OFF = V_OFF + 4 * TILE;     // 2 sub-tiles
constexpr int BAR_OFF = P_OFF + 2 * TILE;
constexpr int SMEM = BAR_OFF + 256 + 1024;
constexpr uint32_t TMEM_COLS = 512, S_COL = 0, O_COL = 256;
}  // namespace attn

__global__ void __launch_bounds__(192, 1)
    attention_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK0,
                     const __grid_constant__ CUtensorMap tmV0, const __grid_constant__ CUtensorMap tmK1,
                     const __grid_constant__ CUtensorMap tmV1, const AttnArgs args) {
  using namespace attn;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;      // [2]
  uint64_t* v_full = bars + 3;      // [2]
  uint64_t* kv_empty = bars + 5;    // [2]
  uint64_t* s_full = bars + 7;      // [2]
  uint64_t* s_free = bars + 9;      // [2]
  uint64_t* p_full = bars + 11;
  uint64_t* o_done = bars + 12;
  uint64_t* drain = bars + 13;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = blockIdx.x * BQ, head = blockIdx.y;
  int n0 = __ldg(args.meta), n1 = __ldg(args.meta + 1);
  n0 = min(max(n0, 0), args.max_keys0);
  n1 = min(max(n1, 0), args.max_keys1);
  const int nb0 = (n0 + BKV - 1) / BKV, nb1 = (n1 + BKV - 1) / BKV, nblk = nb0 + nb1;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(k_full + s, 1);
      mbar_init(v_full + s, 1);
      mbar_init(kv_empty + s, 1);
      mbar_init(s_full + s, 1);
      mbar_init(s_free + s, 128);
    }
    mbar_init(p_full, 128);
    mbar_init(o_done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int col = head * HD;

  if (warp == 4) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0 && nblk > 0) {
      uint32_t used = 0, last_par = 0;
      mbar_arrive_expect_tx(q_full, 2 * TILE);
      tma_load_2d(smem + Q_OFF, &tmQ, q_full, col, q0);
      tma_load_2d(smem + Q_OFF + TILE, &tmQ, q_full, col + 64, q0);
      for (int j = 0; j < nblk; ++j) {
        const int s = j & 1;
        const uint32_t par = (uint32_t)(j >> 1) & 1u;
        if (!mbar_wait(kv_empty + s, par ^ 1u, abort_flag, args.status, DEV_TIMEOUT_PRODUCER)) break;
        const bool seg0 = j < nb0;
        const CUtensorMap* mk = seg0 ? &tmK0 : &tmK1;
        const CUtensorMap* mv = seg0 ? &tmV0 : &tmV1;
        const int key0 = (seg0 ? j : j - nb0) * BKV;
        uint8_t* sk = smem + K_OFF + s * 2 * TILE;
        uint8_t* sv = smem + V_OFF + s * 2 * TILE;
        mbar_arrive_expect_tx(k_full + s, 2 * TILE);
        tma_load_2d(sk, mk, k_full + s, col, key0);
        tma_load_2d(sk + TILE, mk, k_full + s, col + 64, key0);
        mbar_arrive_expect_tx(v_full + s, 2 * TILE);
        tma_load_2d(sv, mv, v_full + s, col, key0);
        tma_load_2d(sv + TILE, mv, v_full + s, col + 64, key0);
        used |= 1u << s;
        last_par = (last_par & ~(1u << s)) | (par << s);
      }
      volatile int no_abort = 0;
      mbar_wait(q_full, 0, &no_abort, args.status, DEV_TIMEOUT_DRAIN);
      for (int s = 0; s < 2; ++s)
        if (used >> s & 1u) {
          mbar_wait(k_full + s, last_par >> s & 1u, &no_abort, args.status, DEV_TIMEOUT_DRAIN);
          mbar_wait(v_full + s, last_par >> s & 1u, &no_abort, args.status, DEV_TIMEOUT_DRAIN);
        }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && nblk > 0) {
      constexpr uint32_t idesc_s = idesc_bf16(128, 128, false, false);   // Q K^T: both K-major
      constexpr uint32_t idesc_o = idesc_bf16(128, 128, false, true);    // P V: V is MN-major
      const uint32_t sq = smem_u32(smem + Q_OFF), sp = smem_u32(smem + P_OFF);
      bool ok = mbar_wait(q_full, 0, abort_flag, args.status, DEV_TIMEOUT_MMA);
      auto issue_s = [&](int j) -> bool {
        const int s = j & 1;
        const uint32_t par = (uint32_t)(j >> 1) & 1u;
        if (!mbar_wait(k_full + s, par, abort_flag, args.status, DEV_TIMEOUT_MMA)) return false;
        if (!mbar_wait(s_free + s, par ^ 1u, abort_flag, args.status, DEV_TIMEOUT_MMA)) return false;
        tc_fence_after();
        const uint32_t sk = smem_u32(smem + K_OFF + s * 2 * TILE);
        const uint32_t d = tmem + S_COL + (uint32_t)(s * 128);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (uint32_t)((kk >> 2) * TILE + (kk & 3) * 32);
          umma_bf16(d, sdesc_sw128(sq + off, 16, 1024), sdesc_sw128(sk + off, 16, 1024), idesc_s, kk != 0);
        }
        umma_commit(s_full + s);
        return true;
      };
      auto issue_o = [&](int j) -> bool {
        const int s = j & 1;
        const uint32_t par = (uint32_t)(j >> 1) & 1u;
        if (!mbar_wait(p_full, (uint32_t)j & 1u, abort_flag, args.status, DEV_TIMEOUT_MMA)) return false;
        if (!mbar_wait(v_full + s, par, abort_flag, args.status, DEV_TIMEOUT_MMA)) return false;
        tc_fence_after();
        const uint32_t sv = smem_u32(smem + V_OFF + s * 2 * TILE);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t aoff = (uint32_t)((kk >> 2) * TILE + (kk & 3) * 32);
          // V sub-tiles hold 64 head-dim columns each (LBO = TILE); 16 keys = 2 atoms of 8 rows.
          umma_bf16(tmem + O_COL, sdesc_sw128(sp + aoff, 16, 1024), sdesc_sw128(sv + (uint32_t)(kk * 2048), TILE, 1024),
                    idesc_o, (j | kk) != 0);
        }
        umma_commit(o_done);
        umma_commit(kv_empty + s);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; ok && j < nblk; ++j) {
        if (j + 1 < nblk) ok = issue_s(j + 1);
        if (ok) ok = issue_o(j);
      }
      umma_commit(drain);
      volatile int no_abort = 0;
      mbar_wait(drain, 0, &no_abort, args.status, DEV_TIMEOUT_DRAIN);
    }
  } else {
    // ------------------------------------------------------------ softmax / correction / epilogue
    const int row = warp * 32 + lane;                       // query row within the tile == TMEM lane
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const float sl2 = args.scale_log2;
    float m = -INFINITY, l = 0.f;
    uint8_t* sP = smem + P_OFF;
    bool ok = true;
    for (int j = 0; j < nblk; ++j) {
      const int s = j & 1;
      const uint32_t par = (uint32_t)(j >> 1) & 1u;
      ok = mbar_wait(s_full + s, par, abort_flag, args.status, DEV_TIMEOUT_SOFTMAX);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      tc_fence_after();
      float sv[128];
      {
        uint32_t r[32];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          tmem_ld32(tmem + lane_off + S_COL + (uint32_t)(s * 128 + c * 32), r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) sv[c * 32 + i] = __uint_as_float(r[i]);
        }
      }
      tc_fence_before();
      mbar_arrive(s_free + s);
      const int valid = (j < nb0) ? min(BKV, n0 - j * BKV) : min(BKV, n1 - (j - nb0) * BKV);
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < 128; ++i) {
        sv[i] = (i < valid) ? sv[i] * sl2 : -INFINITY;
        mx = fmaxf(mx, sv[i]);
      }
      const float m_new = fmaxf(m, mx);
      const float alpha = ex2(m - m_new);   // 0 on the first block (m = -inf)
      float rs = 0.f;
#pragma unroll
      for (int i = 0; i < 128; ++i) {
        sv[i] = ex2(sv[i] - m_new);
        rs += sv[i];
      }
      l = l * alpha + rs;
      m = m_new;
      if (j > 0) {
        ok = mbar_wait(o_done, (uint32_t)(j - 1) & 1u, abort_flag, args.status, DEV_TIMEOUT_SOFTMAX);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha < 1.f)) {
          uint32_t r[32];
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            const uint32_t ta = tmem + lane_off + O_COL + (uint32_t)(c * 32);
            tmem_ld32(ta, r);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
            tmem_st32(ta, r);
          }
          tmem_st_wait();
        }
      }
      // P row -> smem, K-major with the 128-byte swizzle: 16-byte chunk c of row `row` in
      // sub-tile (c / 8) sits at chunk position (c % 8) ^ (row % 8).
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const int sub = c >> 3, ch = c & 7;
        uint4 u = make_uint4(pack_bf16(sv[c * 8 + 0], sv[c * 8 + 1]), pack_bf16(sv[c * 8 + 2], sv[c * 8 + 3]),
                             pack_bf16(sv[c * 8 + 4], sv[c * 8 + 5]), pack_bf16(sv[c * 8 + 6], sv[c * 8 + 7]));
        *reinterpret_cast<uint4*>(sP + sub * TILE + row * 128 + ((ch ^ (row & 7)) << 4)) = u;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok && nblk > 0) {
      ok = mbar_wait(o_done, (uint32_t)(nblk - 1) & 1u, abort_flag, args.status, DEV_TIMEOUT_SOFTMAX);
      if (__all_sync(0xffffffffu, ok)) {
        tc_fence_after();
        const float inv = 1.f / l;
        const int grow = q0 + row;
        uint32_t r[32];
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          tmem_ld32(tmem + lane_off + O_COL + (uint32_t)(c * 32), r);
          tmem_ld_wait();
          if (grow < args.Lq) {
            uint4* dst = reinterpret_cast<uint4*>(args.out + (size_t)grow * args.ld_out + col + c * 32);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              dst[i] = make_uint4(pack_bf16(__uint_as_float(r[8 * i + 0]) * inv, __uint_as_float(r[8 * i + 1]) * inv),
                                  pack_bf16(__uint_as_float(r[8 * i + 2]) * inv, __uint_as_float(r[8 * i + 3]) * inv),
                                  pack_bf16(__uint_as_float(r[8 * i + 4]) * inv, __uint_as_float(r[8 * i + 5]) * inv),
                                  pack_bf16(__uint_as_float(r[8 * i + 6]) * inv, __uint_as_float(r[8 * i + 7]) * inv));
          }
        }
        tc_fence_before();
      }
    }
  }
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

int attention_launch(const CUtensorMap& tmQ, const CUtensorMap& tmK0, const CUtensorMap& tmV0,
                     const CUtensorMap& tmK1, const CUtensorMap& tmV1, const AttnArgs& a, cudaStream_t s) {
  if (a.Lq <= 0 || a.heads <= 0 || !a.meta || !a.out) return FW_EINVAL;
  if (a.ld_out % 8 || (reinterpret_cast<uintptr_t>(a.out) & 15u)) return FW_EALIGN;
  cudaError_t err =
      cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, attn::SMEM);
  if (err != cudaSuccess) return FW_ECUDA;
  dim3 grid((a.Lq + attn::BQ - 1) / attn::BQ, a.heads);
  attention_kernel<<<grid, 192, attn::SMEM, s>>>(tmQ, tmK0, tmV0, tmK1, tmV1, a);
  note_launch();
  return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
}

}  // namespace fw
