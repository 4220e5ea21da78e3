// Flash-style attention forward on tcgen05 for sm_100a (non-causal, head_dim 128).
//
// Replaces flash_attn_varlen_func in the reference forward (fastworld/models/mg2/static.py:
// 138-143): self-attention over [history | current] keys (static.py:213-216) and cross-attention
// over the 257 image-context tokens (static.py:187-192).  Keys come in two segments (the
// per-layer history buffer, then the current chunk) whose lengths are read from device memory,
// so one captured graph serves chunk 0 (no history) and steady chunks, with no host cu_seqlens
// and no concatenation.
//
// One CTA per (pair of 128-query tiles A and B, head); 352 threads:
//   warps 0-3  softmax of tile A, warps 4-7 softmax of tile B: thread = query row (TMEM lane).
//              Loads its S row from TMEM, online softmax in the exp2 domain (1/16 of the
//              exponentials by a polynomial on the FMA pipe, the rest on the SFU) with a lazy O
//              rescale (only when the running max grows by more than 2^8), writes P (bf16)
//              into its tile's 128-byte-swizzled K-major smem buffer, final O / l and store.
//   warp 8     TMA producer: both Q tiles once; then K_0, V_0, K_1, V_1, ... through a ring of
//              three 32 KB slots (K_{j+1} lands while V_j is still in use).
//   warps 9-10 MMA issuers, one per tile, so the tensor core interleaves the tiles' work and
//              a slow softmax on one tile never holds back the other:
//                S_t(j+1) = Q_t K_{j+1}^T,  O_t += P_t(j) V_j;  K/V ring slots are released once
//              both tiles committed their reads.
// TMEM (512 columns): S_A [0,128), O_A [128,256), S_B [256,384), O_B [384,512).
// SMEM: Q_A, Q_B (2 x 32 KB), K/V ring (3 x 32 KB), P_A, P_B (2 x 32 KB) = 224 KB.
#include "../../include/fastworld_b200.h"
#include "fw_internal.h"
#include "fw_ptx.cuh"

namespace fw {

namespace attn {
constexpr int BQ = 128, BKV = 128, HD = 128;
constexpr int THREADS = 352;
constexpr int TILE = 128 * 64 * 2;          // one [128 rows x 64 cols] bf16 swizzled sub-tile (16 KB)
constexpr int Q_OFF = 0;                    // tile t: 2 sub-tiles at Q_OFF + t * 2 * TILE
constexpr int KV_OFF = Q_OFF + 4 * TILE;    // slot s: 2 sub-tiles at KV_OFF + s * 2 * TILE
constexpr int P_OFF = KV_OFF + 6 * TILE;    // tile t: 2 sub-tiles at P_OFF + t * 2 * TILE
constexpr int BAR_OFF = P_OFF + 4 * TILE;
constexpr int SMEM = BAR_OFF + 256 + 1024;
constexpr uint32_t TMEM_COLS = 512;
// Tile B's first S MMA waits until tile A's softmax of block 0 has started, so the two tiles'
// softmax phases and MMA phases interleave instead of coinciding (measured at the MG2 steady
// shape: 89.6 us against 93.7 us for a simultaneous start, 91.4 us when tile B waits for tile
// A's whole first softmax and 91.0 us when it waits for its exponentials).
constexpr bool STAGGER = true;
// Load order through the K/V ring: K0, K1, V0, K2, V1, K3, V2, ..., K_{n-1}, V_{n-2}, V_{n-1}
// (the order the MMA issuers consume them: S(0), S(1), PV(0), S(2), PV(1), ...), so each K
// block is loaded one block further ahead than its V.  Position of each load in that sequence:
__host__ __device__ constexpr int pos_k(int j) { return j == 0 ? 0 : 2 * j - 1; }
__host__ __device__ constexpr int pos_v(int j, int n) { return 2 * j + 2 < 2 * n - 1 ? 2 * j + 2 : 2 * n - 1; }
__host__ __device__ constexpr uint32_t s_col(int t) { return (uint32_t)(t * 256); }
__host__ __device__ constexpr uint32_t o_col(int t) { return (uint32_t)(t * 256 + 128); }
}  // namespace attn

__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x on the FMA pipe (x <= 8; clamped to >= -125, where 2^x is below any weight that counts):
// x = n + f with n = round(x) by the 1.5 * 2^23 shifter (FADD, no conversion instruction) and
// f in [-0.5, 0.5]; 2^f by a degree-3 polynomial whose coefficients were fitted to minimise the
// relative error on [-0.5, 0.5] (Lawson's iteration; 7.5e-5 in fp32 Horner form, far below the
// 2^-9 rounding of the bf16 P it feeds); 2^n added to the exponent field (n << 23 is the
// shifter's bits << 23).  Two lanes per call on the packed fp32 pipe.
__device__ __forceinline__ float2 ex2_fma2(float2 x) {
  x.x = fmaxf(x.x, -125.f);
  x.y = fmaxf(x.y, -125.f);
  const float2 t = __fadd2_rn(x, make_float2(12582912.f, 12582912.f));
  const float2 nf = __fadd2_rn(t, make_float2(-12582912.f, -12582912.f));
  const float2 f = __ffma2_rn(nf, make_float2(-1.f, -1.f), x);
  float2 p = __ffma2_rn(make_float2(0.05517132207751274f, 0.05517132207751274f), f,
                        make_float2(0.24261054396629333f, 0.24261054396629333f));
  p = __ffma2_rn(p, f, make_float2(0.6932609677314758f, 0.6932609677314758f));
  p = __ffma2_rn(p, f, make_float2(0.9999281167984009f, 0.9999281167984009f));
  return make_float2(__int_as_float(__float_as_int(p.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(p.y) + (__float_as_int(t.y) << 23)));
}

// TMA_OUT: O leaves through the tile's (then idle) P buffer with two TMA stores per tile instead
// of each softmax thread storing its own row (32 rows per warp store instruction).
template <bool TMA_OUT>
__global__ void __launch_bounds__(attn::THREADS, 1)
    attention_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK0,
                     const __grid_constant__ CUtensorMap tmV0, const __grid_constant__ CUtensorMap tmK1,
                     const __grid_constant__ CUtensorMap tmV1, const __grid_constant__ CUtensorMap tmO,
                     const AttnArgs args) {
  using namespace attn;
  pdl_trigger();
  pdl_wait();
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;     // [3] ring slots
  uint64_t* kv_free = bars + 4;     // [3]
  uint64_t* s_full = bars + 7;      // [2] per tile
  uint64_t* s_free = bars + 9;      // [2]
  uint64_t* p_full = bars + 11;     // [2]
  uint64_t* o_done = bars + 13;     // [2]
  uint64_t* drain = bars + 15;       // [tile 0]; tile 1 uses bars + 17
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = blockIdx.x * 2 * BQ, head = blockIdx.y;
  const int ntile = (q0 + BQ < args.Lq) ? 2 : 1;   // tile B exists only if it has query rows
  int n0 = __ldg(args.meta), n1 = __ldg(args.meta + 1);
  n0 = min(max(n0, 0), args.max_keys0);
  n1 = min(max(n1, 0), args.max_keys1);
  const int nb0 = (n0 + BKV - 1) / BKV, nb1 = (n1 + BKV - 1) / BKV, nblk = nb0 + nb1;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 3; ++s) {
      mbar_init(kv_full + s, 1);
      mbar_init(kv_free + s, ntile);   // released once every tile's MMAs read the slot
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(s_full + t, 1);
      mbar_init(s_free + t, 128);
      mbar_init(p_full + t, 128);
      mbar_init(o_done + t, 1);
    }
    mbar_init(drain, 1);
    mbar_init(bars + 17, 1);
    mbar_init(bars + 18, 1);   // stagger: tile A's softmax has started (once)
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int col = head * HD;

  if (warp == 8) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0 && nblk > 0) {
      uint32_t used = 0, last_par = 0;
      mbar_arrive_expect_tx(q_full, ntile * 2 * TILE);
      for (int t = 0; t < ntile; ++t) {
        tma_load_2d(smem + Q_OFF + t * 2 * TILE, &tmQ, q_full, col, q0 + t * BQ);
        tma_load_2d(smem + Q_OFF + t * 2 * TILE + TILE, &tmQ, q_full, col + 64, q0 + t * BQ);
      }
      for (int i = 0; i < 2 * nblk; ++i) {   // load at position i of the order above
        const int s = i % 3;
        const uint32_t par = (uint32_t)(i / 3) & 1u;
        if (!mbar_wait(kv_free + s, par ^ 1u, abort_flag, args.status, DEV_TIMEOUT_PRODUCER)) break;
        bool is_v;
        int j;
        if (i == 0) {
          is_v = false, j = 0;
        } else if (i == 2 * nblk - 1) {
          is_v = true, j = nblk - 1;
        } else if (i & 1) {
          is_v = false, j = (i + 1) >> 1;
        } else {
          is_v = true, j = (i - 2) >> 1;
        }
        const bool seg0 = j < nb0;
        const CUtensorMap* m = is_v ? (seg0 ? &tmV0 : &tmV1) : (seg0 ? &tmK0 : &tmK1);
        const int key0 = (seg0 ? j : j - nb0) * BKV;
        uint8_t* dst = smem + KV_OFF + s * 2 * TILE;
        mbar_arrive_expect_tx(kv_full + s, 2 * TILE);
        tma_load_2d(dst, m, kv_full + s, col, key0);
        tma_load_2d(dst + TILE, m, kv_full + s, col + 64, key0);
        used |= 1u << s;
        last_par = (last_par & ~(1u << s)) | (par << s);
      }
      volatile int no_abort = 0;
      mbar_wait(q_full, 0, &no_abort, args.status, DEV_TIMEOUT_DRAIN);
      for (int s = 0; s < 3; ++s)
        if (used >> s & 1u) mbar_wait(kv_full + s, last_par >> s & 1u, &no_abort, args.status, DEV_TIMEOUT_DRAIN);
    }
  } else if (warp == 9 || warp == 10) {
    // ------------------------------------------------------------ MMA issuers (one per tile)
    const int tt = warp - 9;
    if (lane == 0 && nblk > 0 && tt < ntile) {
      constexpr uint32_t idesc_s = idesc_bf16(128, 128, false, false);   // Q K^T: both K-major
      constexpr uint32_t idesc_o = idesc_bf16(128, 128, false, true);    // P V: V is MN-major
      bool ok = mbar_wait(q_full, 0, abort_flag, args.status, DEV_TIMEOUT_MMA);
      // S_t(j) = Q_t K_j^T into the tile's S columns; needs K_j landed and S_t(j-1) read out
      auto issue_s = [&](int t, int j) -> bool {
        const int pk = pos_k(j), s = pk % 3;
        if (!mbar_wait(kv_full + s, (uint32_t)(pk / 3) & 1u, abort_flag, args.status, DEV_TIMEOUT_MMA))
          return false;
        if (!mbar_wait(s_free + t, ((uint32_t)j & 1u) ^ 1u, abort_flag, args.status, DEV_TIMEOUT_MMA)) return false;
        tc_fence_after();
        const uint32_t sq = smem_u32(smem + Q_OFF + t * 2 * TILE);
        const uint32_t sk = smem_u32(smem + KV_OFF + s * 2 * TILE);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (uint32_t)((kk >> 2) * TILE + (kk & 3) * 32);
          umma_bf16(tmem + s_col(t), sdesc_sw128(sq + off, 16, 1024), sdesc_sw128(sk + off, 16, 1024), idesc_s,
                    kk != 0);
        }
        umma_commit(s_full + t);
        umma_commit(kv_free + s);   // this tile is done with K_j
        return true;
      };
      // O_t += P_t(j) V_j; needs P_t(j) written and V_j landed
      auto issue_o = [&](int t, int j) -> bool {
        const int pv = pos_v(j, nblk), s = pv % 3;
        if (!mbar_wait(p_full + t, (uint32_t)j & 1u, abort_flag, args.status, DEV_TIMEOUT_MMA)) return false;
        if (!mbar_wait(kv_full + s, (uint32_t)(pv / 3) & 1u, abort_flag, args.status, DEV_TIMEOUT_MMA))
          return false;
        tc_fence_after();
        const uint32_t sp = smem_u32(smem + P_OFF + t * 2 * TILE);
        const uint32_t sv = smem_u32(smem + KV_OFF + s * 2 * TILE);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t aoff = (uint32_t)((kk >> 2) * TILE + (kk & 3) * 32);
          // V sub-tiles hold 64 head-dim columns each (LBO = TILE); 16 keys = 2 atoms of 8 rows.
          umma_bf16(tmem + o_col(t), sdesc_sw128(sp + aoff, 16, 1024),
                    sdesc_sw128(sv + (uint32_t)(kk * 2048), TILE, 1024), idesc_o, (j | kk) != 0);
        }
        umma_commit(o_done + t);
        umma_commit(kv_free + s);   // this tile is done with V_j
        return true;
      };
      if (ok && tt == 1 && STAGGER) {   // start tile B behind tile A
        ok = mbar_wait(bars + 18, 0, abort_flag, args.status, DEV_TIMEOUT_MMA);
      }
      if (ok) ok = issue_s(tt, 0);
      for (int j = 0; ok && j < nblk; ++j) {
        if (j + 1 < nblk) ok = issue_s(tt, j + 1);
        if (ok) ok = issue_o(tt, j);
      }
      uint64_t* my_drain = tt == 0 ? drain : bars + 17;
      umma_commit(my_drain);
      volatile int no_abort = 0;
      mbar_wait(my_drain, 0, &no_abort, args.status, DEV_TIMEOUT_DRAIN);
    }
  } else if ((warp >> 2) < ntile) {
    // ------------------------------------------------------------ softmax / correction / epilogue
    const int t = warp >> 2, q = warp & 3;
    const int row = q * 32 + lane;                            // query row within the tile == TMEM lane
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const float sl2 = args.scale_log2;
    float m = -INFINITY, l = 0.f;
    uint8_t* sP = smem + P_OFF + t * 2 * TILE;
    bool ok = true;
    for (int j = 0; j < nblk; ++j) {
      ok = mbar_wait(s_full + t, (uint32_t)j & 1u, abort_flag, args.status, DEV_TIMEOUT_SOFTMAX);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      tc_fence_after();
      float sv[128];
      {
        uint32_t* r = reinterpret_cast<uint32_t*>(sv);
#pragma unroll
        for (int c = 0; c < 4; ++c)
          tmem_ld32(tmem + lane_off + s_col(t) + (uint32_t)(c * 32), *reinterpret_cast<uint32_t(*)[32]>(r + 32 * c));
        tmem_ld_wait();
      }
      tc_fence_before();
      mbar_arrive(s_free + t);
      if (STAGGER && j == 0 && t == 0 && threadIdx.x == 0) mbar_arrive(bars + 18);
      const int valid = (j < nb0) ? min(BKV, n0 - j * BKV) : min(BKV, n1 - (j - nb0) * BKV);
      if (valid < BKV) {   // ragged last block of a segment
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i >= valid) sv[i] = -INFINITY;
      }
      // row max with three-input max (64 instructions for 128 scores)
      float mx8[8];
#pragma unroll
      for (int a = 0; a < 8; ++a) mx8[a] = fmaxf(sv[a], sv[a + 8]);
#pragma unroll
      for (int i = 16; i < 128; i += 16)
#pragma unroll
        for (int a = 0; a < 8; ++a) mx8[a] = max3f(mx8[a], sv[i + a], sv[i + 8 + a]);
      const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                             fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]))) * sl2;
      // lazy rescale: keep the running max unless it grows by more than 2^8 (p stays <= 256)
      float alpha = 1.f;
      if (mx > m + 8.f) {
        alpha = ex2(m - mx);   // 0 on the first block (m = -inf)
        m = mx;
      }
      // exponent arguments and row sums on packed fp32 pairs (half the FFMA / FADD instructions);
      // rs2[c] holds the sums of elements 8k + 2c and 8k + 2c + 1, in ascending k
      float2 rs2[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) rs2[c] = make_float2(0.f, 0.f);
      const float2 sl2v = make_float2(sl2, sl2), nm = make_float2(-m, -m);
#pragma unroll
      for (int j = 0; j < 64; ++j) {
        const float2 x = __ffma2_rn(make_float2(sv[2 * j], sv[2 * j + 1]), sl2v, nm);
        // four of the 64 pairs (1/16 of the exponentials) on the FMA pipe; measured at the MG2
        // steady shape: 87.8 -> 82.0 us (1/32: 85.9, 1/8: 83.0, 1/4: 86.8, a third: 89.0)
        if ((j & 15) == 15) {
          const float2 e = ex2_fma2(x);
          sv[2 * j] = e.x;
          sv[2 * j + 1] = e.y;
        } else {
          sv[2 * j] = ex2(x.x);
          sv[2 * j + 1] = ex2(x.y);
        }
        rs2[j & 3] = __fadd2_rn(rs2[j & 3], make_float2(sv[2 * j], sv[2 * j + 1]));
      }
      l = l * alpha + (((rs2[0].x + rs2[0].y) + (rs2[1].x + rs2[1].y)) + ((rs2[2].x + rs2[2].y) + (rs2[3].x + rs2[3].y)));
      if (j > 0) {   // P buffer and O are free once the previous P V finished
        ok = mbar_wait(o_done + t, (uint32_t)(j - 1) & 1u, abort_flag, args.status, DEV_TIMEOUT_SOFTMAX);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha < 1.f)) {
          uint32_t r[32];
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            const uint32_t ta = tmem + lane_off + o_col(t) + (uint32_t)(c * 32);
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
      mbar_arrive(p_full + t);
    }
    if (ok && nblk > 0) {
      ok = mbar_wait(o_done + t, (uint32_t)(nblk - 1) & 1u, abort_flag, args.status, DEV_TIMEOUT_SOFTMAX);
      if (__all_sync(0xffffffffu, ok)) {
        tc_fence_after();
        const float inv = 1.f / l;
        const int grow = q0 + t * BQ + row;
        uint32_t r[32];
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          tmem_ld32(tmem + lane_off + o_col(t) + (uint32_t)(c * 32), r);
          tmem_ld_wait();
          uint4 u[4];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            u[i] = make_uint4(pack_bf16(__uint_as_float(r[8 * i + 0]) * inv, __uint_as_float(r[8 * i + 1]) * inv),
                              pack_bf16(__uint_as_float(r[8 * i + 2]) * inv, __uint_as_float(r[8 * i + 3]) * inv),
                              pack_bf16(__uint_as_float(r[8 * i + 4]) * inv, __uint_as_float(r[8 * i + 5]) * inv),
                              pack_bf16(__uint_as_float(r[8 * i + 6]) * inv, __uint_as_float(r[8 * i + 7]) * inv));
          if constexpr (TMA_OUT) {   // into the P buffer (its last reader, the final P V, completed)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int chunk = c * 4 + i, sub = chunk >> 3, ch = chunk & 7;
              *reinterpret_cast<uint4*>(sP + sub * TILE + row * 128 + ((ch ^ (row & 7)) << 4)) = u[i];
            }
          } else if (grow < args.Lq) {
            uint4* dst = reinterpret_cast<uint4*>(args.out + (size_t)grow * args.ld_out + col + c * 32);
#pragma unroll
            for (int i = 0; i < 4; ++i) dst[i] = u[i];
          }
        }
        if constexpr (TMA_OUT) fence_proxy_async_smem();
        tc_fence_before();
      }
    }
    if constexpr (TMA_OUT) {
      // the tile's 128 softmax threads meet (named barrier 1 + t), then one stores the tile: rows
      // past Lq are clipped by the tensor map
      if (t == 0)
        asm volatile("bar.sync 1, 128;" ::: "memory");
      else
        asm volatile("bar.sync 2, 128;" ::: "memory");
      if (q == 0 && lane == 0 && ok && nblk > 0) {
        tma_store_2d(&tmO, sP, col, q0 + t * BQ);
        tma_store_2d(&tmO, sP + TILE, col + 64, q0 + t * BQ);
        bulk_commit();
        bulk_wait0();
      }
    }
  }
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

int attention_launch(const CUtensorMap& tmQ, const CUtensorMap& tmK0, const CUtensorMap& tmV0,
                     const CUtensorMap& tmK1, const CUtensorMap& tmV1, const AttnArgs& a, cudaStream_t s,
                     const CUtensorMap* tmO) {
  if (a.Lq <= 0 || a.heads <= 0 || !a.meta || !a.out) return FW_EINVAL;
  if (a.ld_out % 8 || (reinterpret_cast<uintptr_t>(a.out) & 15u)) return FW_EALIGN;
  dim3 grid((a.Lq + 2 * attn::BQ - 1) / (2 * attn::BQ), a.heads);
  auto go = [&](auto kern, const CUtensorMap& o) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, attn::SMEM) != cudaSuccess)
      return FW_ECUDA;
    launch_k(kern, grid, attn::THREADS, attn::SMEM, s, tmQ, tmK0, tmV0, tmK1, tmV1, o, a);
    return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
  };
  return tmO ? go(attention_kernel<true>, *tmO) : go(attention_kernel<false>, tmQ);
}

}  // namespace fw
