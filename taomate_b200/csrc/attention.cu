// Block-causal streaming attention on sm_100a tensor cores.
//
// Each CTA runs two softmax warpgroups ("lanes") over the ordered list of
// visible 64-key tiles (anchor + rolling window from the slot arena, then the
// current chunk) of one (batch, head):
//   pair CTA:  lane l owns query tile 2c + l; both lanes consume every K/V tile,
//              so a tile is loaded once for 256 query rows.
//   split CTA: the odd last query tile of a head; both lanes use the same Q,
//              lane 0 takes the first ceil(n/2) key tiles and lane 1 the rest,
//              and lane 0 merges the two partial results.  Split CTAs come
//              after the pair CTAs in grid order, so they fill the tail of the
//              wave.
// When pair CTAs would leave SMs idle (few heads per GPU under sequence
// parallelism, or a short query chunk), every CTA is a split CTA for one
// query tile, and with a workspace the key tiles are further divided into
// kv_splits ranges, one CTA each; those CTAs write normalised fp32 partial
// outputs with their (max, sum), and a combine kernel merges the ranges.
// The same partial outputs can be exported instead (tm_attention_fwd_ext with
// `parts`): each of several GPUs attends over its own share of the keys, the
// partials are gathered, and tm_attention_combine merges them (V2A under
// sequence parallelism: 25 audio queries over keys split by rank).
//
// Shared memory: the query tile(s) (TMA, 128-byte swizzle), a 4-stage K ring
// and a 5-stage V ring of 64-key tiles.  TMEM (512 columns): S_l at 64 l
// (fp32), P_l double-buffered at 128 + 64 l + 32 b (bf16 pairs), O_l at
// 256 + D l.  S_l = Q_l K^T takes both operands from shared memory; O_l += P_l V
// takes P from TMEM.
//
// Warp roles (12 warps):
//   warp 0      TMA producer of Q and of the K ring (plain tile loads).
//   warp 2      TMA producer of the V ring.
//   warp 1 / 3  tcgen05.mma issuers of lane 0 / lane 1, one thread each: a
//               single thread issues at most one MMA every ~50 cycles, so a
//               64-wide MMA (32 cycles of tensor work) needs two issuers to
//               keep the tensor core busy.  Per lane the order is QK(j),
//               PV(j - 1), QK(j + 1), ...: QK(j + 1) only needs softmax to
//               have read S(j), so it overlaps softmax(j) and PV(j).
//   warps 4..7  lane 0, warps 8..11 lane 1: thread r owns query row r (its TMEM
//               lane); reads its S row, keeps running max / sum in registers,
//               writes P (bf16) into TMEM, rescales O only when its running
//               max grows by more than 2^8 (the final division uses the same
//               reference max).  A fixed share of the exponentials runs on the
//               FMA pipe (Cody-Waite split 2^x = 2^round(x) * 2^f, |f| <= 1/2,
//               degree-3 minimax polynomial for 2^f, max relative error
//               7.5e-5).
//
// Visibility (anchor + window + chunk) arrives as a host-built list of key
// tiles (source, first row, valid rows); keys beyond `valid` are masked to
// -inf in registers, nothing is materialised.
//
// Reference semantics: softmax(Q K^T / sqrt(D)) V without a mask over
// cat(cached, new) (ltx_causal/transformer/kv_cache.py:1486-1531,
// ltx_causal/attention/flex_attention_utils.py:225-276).
#include <algorithm>
#include <climits>
#include <cmath>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "host_common.h"

namespace tmb {
namespace attn {

constexpr int BM = 128;          // query rows per lane (one TMEM lane each)
constexpr int BN = 64;           // keys per tile
constexpr int kMaxTiles = 384;   // 24576 visible keys
constexpr int kThreads = 384;    // 12 warps
// Register split (setmaxnreg): launched at 168 per thread (384 x 168 =
// 64512); warpgroup 0 drops to 88, the two softmax warpgroups rise to 208:
// 128 x 88 + 256 x 208 = 64512, the launch total.
constexpr int kRegsCtrl = 88;
constexpr int kRegsSoftmax = 208;
// Exponentials on the FMA pipe: kEmulPairs of every 4 column pairs.
constexpr int kEmulPairs = 1;

struct __align__(64) Params {
  float* part_o;          // kv_splits > 1: [kv_splits][B][Lq][H][D] normalised partial outputs
  float2* part_ml;        //                [kv_splits][B][Lq][H] (max * log2 scale, sum)
  const int2* tiles_dev;  // non-null: read the key-tile list from device memory (graph replay)
  int mode;               // 0: pair CTAs (+ one split CTA for an odd tile); 1: split CTAs only;
                          // 2: pair CTAs, the odd tiles of heads (h, h + 1) in one CTA
  int kv_splits;          // mode 1: key-tile ranges per query tile
  int partial_only;       // part_o / part_ml belong to the caller: no combine pass
  CUtensorMap tm_q;
  CUtensorMap tm_k[2];  // [TM_KV_SOURCE_CACHE], [TM_KV_SOURCE_NEW]
  CUtensorMap tm_v[2];
  int2 tiles[kMaxTiles];  // x = (source << 30) | first row, y = valid rows (1..BN)
  int n_tiles;
  int n_qtiles;            // ceil(Lq / BM)
  int Lq;
  int64_t out_bs, out_rs;  // elements
  __nv_bfloat16* out;
  // Output row placement: query row r goes to rank r / rows_per_rank, local
  // row r % rows_per_rank, head head_base + h, at `out` + out_delta[rank]
  // bytes (peer buffers mapped into this process; 0 for this rank).
  int rows_per_rank;
  int head_base;
  int64_t out_delta[8];
  int stage_out;  // some rows go to another rank: store whole rows through shared memory
  // Per-head output gate 2 * sigmoid(logit), logits [B, Lq, H] bf16 (head
  // stride 1), or null.
  const __nv_bfloat16* gate;
  int64_t gate_bs, gate_rs;
  float scale_log2;
  int* err;
};

template <int D>
struct Cfg {
  static constexpr int kKStages = 4;
  static constexpr int kVStages = 5;
  static constexpr int kBlk = BN * 128;   // one 64-key x 64-column swizzle block of K / V
  static constexpr int kQBlk = BM * 128;  // one 128-row x 64-column block of Q
  static constexpr int kQBytes = BM * D * 2;
  static constexpr int kKVBytes = BN * D * 2;
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + 2 * kQBytes;
  static constexpr int kVOff = kKOff + kKStages * kKVBytes;
  static constexpr int kBarOff = kVOff + kVStages * kKVBytes;
  // barriers: q_full, k_full[KS], k_empty[KS], v_full[VS], v_empty[VS],
  //           s_full[2][2], p_full[2][2], pv_done[2][2], drain[2]
  static constexpr int kNumBars = 1 + 2 * kKStages + 2 * kVStages + 14;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;  // tmem slot, abort flag
  static constexpr int kMLOff = kMiscOff + 16;             // lane-1 max / sum per row
  static constexpr int kSmemBytes = kMLOff + 2 * BM * 4;
  static constexpr int kSmemAlloc = kSmemBytes + 1024;     // runtime 1 KB alignment slack
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kSCol = 0;     // S_l,b at kSCol + 128 l + 64 b; P over its first 32
  static constexpr uint32_t kOCol = 256;   // O_l at kOCol + D l
};

// 2^x on the FMA / ALU pipes for two values: x clamped to >= -126, split as
// round(x) + f, 2^f from a degree-3 minimax polynomial, exponent added in the
// integer domain.
__device__ __forceinline__ void exp2_poly2(float x0, float x1, float& y0, float& y1) {
  const uint64_t kMagic = f2_packf(12582912.0f, 12582912.0f);   // 1.5 * 2^23
  const uint64_t kNegMagic = f2_packf(-12582912.0f, -12582912.0f);
  const uint64_t kNegOne = f2_packf(-1.0f, -1.0f);
  const uint64_t c0 = f2_packf(0.99992806f, 0.99992806f);
  const uint64_t c1 = f2_packf(0.69326097f, 0.69326097f);
  const uint64_t c2 = f2_packf(0.24261114f, 0.24261114f);
  const uint64_t c3 = f2_packf(0.05517167f, 0.05517167f);
  const uint64_t xc = f2_packf(fmaxf(x0, -126.0f), fmaxf(x1, -126.0f));
  const uint64_t t = f2_add(xc, kMagic);      // round(x) in the low mantissa bits
  const uint64_t r = f2_add(t, kNegMagic);    // round(x) as a float
  const uint64_t f = f2_fma(r, kNegOne, xc);  // x - round(x), in [-0.5, 0.5]
  uint64_t pp = f2_fma(f, c3, c2);
  pp = f2_fma(pp, f, c1);
  pp = f2_fma(pp, f, c0);
  float t0, t1, p0, p1;
  f2_unpack(t, t0, t1);
  f2_unpack(pp, p0, p1);
  y0 = __uint_as_float(__float_as_uint(p0) + (__float_as_uint(t0) << 23));
  y1 = __uint_as_float(__float_as_uint(p1) + (__float_as_uint(t1) << 23));
}

// 2 * sigmoid of the row's gate logit (1 without a gate).
__device__ __forceinline__ float gate_of(const __nv_bfloat16* gate, int64_t gbs, int64_t grs,
                                         int batch, int qi, int head) {
  if (!gate) return 1.0f;
  const float z = __bfloat162float(gate[static_cast<int64_t>(batch) * gbs +
                                        static_cast<int64_t>(qi) * grs + head]);
  return 2.0f / (1.0f + __expf(-z));
}

// Address of output row qi, head `head`, column 0.
__device__ __forceinline__ __nv_bfloat16* out_row(__nv_bfloat16* out, int64_t out_bs,
                                                  int64_t out_rs, int rows_per_rank,
                                                  int head_base, const int64_t* delta, int batch,
                                                  int qi, int head, int D) {
  int rr = qi / rows_per_rank;
  rr = rr < 0 ? 0 : (rr > 7 ? 7 : rr);
  const int li = qi - rr * rows_per_rank;
  return reinterpret_cast<__nv_bfloat16*>(
      reinterpret_cast<char*>(out + static_cast<int64_t>(batch) * out_bs +
                              static_cast<int64_t>(li) * out_rs +
                              static_cast<int64_t>(head_base + head) * D) +
      delta[rr]);
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1) attn_fwd_kernel(const __grid_constant__ Params p) {
  using C = Cfg<D>;
  constexpr int KS = C::kKStages;
  constexpr int VS = C::kVStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_addr(smem);
  const int warp = threadIdx.x >> 5;
  const int lane_id = threadIdx.x & 31;
  const int head = blockIdx.x, cta = blockIdx.y, batch = blockIdx.z;
  const int n = p.n_tiles;
  const int pairs = p.n_qtiles >> 1;
  const bool single = p.mode == 1;
  // Mode 2: the odd query tile of heads (h, h + 1), h even, in one CTA with one
  // head per lane; the CTA of head h + 1 has nothing to do.  (With an odd head
  // count the last head's odd tile stays a split CTA.)
  const bool odd_tile_cta = !single && cta >= pairs;
  if (p.mode == 2 && odd_tile_cta && (head & 1)) return;
  const bool xh = p.mode == 2 && odd_tile_cta && head + 1 < static_cast<int>(gridDim.x);
  const int kvs = single ? p.kv_splits : 1;
  const int sidx = single ? cta % kvs : 0;  // key range of this CTA
  const bool split = !xh && (single || cta >= pairs);
  const bool alt = split || xh;  // the lanes take alternate items of the K/V stream
  const int qt0 = single ? cta / kvs : 2 * cta;
  // this CTA's key tiles [kb, kb + nr)
  const int kb = static_cast<int>(static_cast<int64_t>(sidx) * n / kvs);
  const int nr = static_cast<int>(static_cast<int64_t>(sidx + 1) * n / kvs) - kb;
  // key tiles per lane; split: lane 0 [kb, kb + n0), lane 1 the rest; pair and
  // cross-head: both all (cross-head: each its own head's copy of the tiles)
  const int n0 = split ? (nr + 1) >> 1 : nr;
  const int n1 = split ? nr - n0 : nr;
  const int n_items = xh ? 2 * nr : nr;  // K/V tile loads of this CTA

  const uint32_t bar0 = sbase + C::kBarOff;
  const uint32_t b_qfull = bar0;
  auto b_kfull = [&](int s) { return bar0 + 8u * (1 + s); };
  auto b_kempty = [&](int s) { return bar0 + 8u * (1 + KS + s); };
  auto b_vfull = [&](int s) { return bar0 + 8u * (1 + 2 * KS + s); };
  auto b_vempty = [&](int s) { return bar0 + 8u * (1 + 2 * KS + VS + s); };
  const uint32_t bar1 = bar0 + 8u * (1 + 2 * KS + 2 * VS);
  auto b_sfull = [&](int l, int b) { return bar1 + 8u * (2 * l + b); };
  auto b_pfull = [&](int l, int b) { return bar1 + 8u * (4 + 2 * l + b); };
  auto b_pvdone = [&](int l, int b) { return bar1 + 8u * (8 + 2 * l + b); };
  auto b_drain = [&](int l) { return bar1 + 8u * (12 + l); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kMiscOff + 4);
  float* m1_smem = reinterpret_cast<float*>(smem + C::kMLOff);
  float* l1_smem = m1_smem + BM;

  // stream item -> key tile (and head, cross-head); lane step -> stream item
  const int2* tl = p.tiles_dev ? p.tiles_dev : p.tiles;
  auto tile_of = [&](int g) {
    if (xh) return kb + (g >> 1);
    return kb + (split ? ((g & 1) ? n0 + (g >> 1) : (g >> 1)) : g);
  };
  auto item_of = [&](int l, int j) { return alt ? 2 * j + l : j; };

  if (threadIdx.x == 0) {
    const uint32_t consumers = alt ? 1u : 2u;
    mbar_init(b_qfull, 1);
    for (int s = 0; s < KS; ++s) {
      mbar_init(b_kfull(s), 1);
      mbar_init(b_kempty(s), consumers);
    }
    for (int s = 0; s < VS; ++s) {
      mbar_init(b_vfull(s), 1);
      mbar_init(b_vempty(s), consumers);
    }
    for (int l = 0; l < 2; ++l) {
      for (int b = 0; b < 2; ++b) {
        mbar_init(b_sfull(l, b), 1);
        mbar_init(b_pfull(l, b), 128);
        mbar_init(b_pvdone(l, b), 1);
      }
      mbar_init(b_drain(l), 1);
    }
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_addr(tmem_slot), C::kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane_id == 0) {
    tma_prefetch_desc(&p.tm_q);
    tma_prefetch_desc(&p.tm_k[0]);
    tma_prefetch_desc(&p.tm_k[1]);
    tma_prefetch_desc(&p.tm_v[0]);
    tma_prefetch_desc(&p.tm_v[1]);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsCtrl));

  if (warp == 0 || warp == 2) {
    // ------------------------------------------------------------------ producers
    if (lane_id == 0) {
      constexpr int kDB = D / 64;
      const bool is_k = warp == 0;
      const int S = is_k ? KS : VS;
      if (is_k) {
        const int nq = split ? 1 : 2;
        mbar_arrive_expect_tx(b_qfull, nq * C::kQBytes);
        for (int t = 0; t < nq; ++t)
          for (int db = 0; db < kDB; ++db)
            tma_load_4d(sbase + C::kQOff + t * C::kQBytes + db * C::kQBlk, &p.tm_q, b_qfull,
                        db * 64, xh ? head + t : head, (xh ? qt0 : qt0 + t) * BM, batch);
      }
      int last = -1;
      for (int g = 0; g < n_items; ++g) {
        const int s = g % S;
        if (g >= S && !mbar_wait(is_k ? b_kempty(s) : b_vempty(s), ((g / S) - 1) & 1, abort_flag,
                                 p.err))
          break;
        const int2 tile = tl[tile_of(g)];
        const int src = tile.x >> 30;
        const int row = tile.x & 0x3FFFFFFF;
        const uint32_t full = is_k ? b_kfull(s) : b_vfull(s);
        const uint32_t dst = sbase + (is_k ? C::kKOff : C::kVOff) + s * C::kKVBytes;
        const CUtensorMap* map = is_k ? &p.tm_k[src] : &p.tm_v[src];
        mbar_arrive_expect_tx(full, C::kKVBytes);
        const int hd = xh ? head + (g & 1) : head;
        for (int db = 0; db < kDB; ++db)
          tma_load_4d(dst + db * C::kBlk, map, full, db * 64, hd, row, batch);
        last = g;
      }
      if (*abort_flag) {
        // Let every issued copy land before the CTA's shared memory is released.
        if (is_k) mbar_wait(b_qfull, 0, nullptr, p.err, 100000000ull);
        for (int g = last - S + 1; g <= last; ++g)
          if (g >= 0)
            mbar_wait(is_k ? b_kfull(g % S) : b_vfull(g % S), (g / S) & 1, nullptr, p.err,
                      100000000ull);
      }
    }
  } else if (warp == 1 || warp == 3) {
    // ------------------------------------------------------------------ MMA issuers
    // The whole warp runs the loop (waits, descriptor arithmetic) so that
    // every value stays warp-uniform; one elected lane issues the MMAs and
    // their commits.
    const int l = warp == 1 ? 0 : 1;
    const int nl = l == 0 ? n0 : n1;
    if (nl > 0) {
      constexpr uint32_t idesc_qk = idesc_bf16_f32(BM, BN, 0);
      constexpr uint32_t idesc_pv = idesc_bf16_f32(BM, D, 1);
      const bool leader = elect_one();
      const int qsel = split ? 0 : l;
      // Descriptors are built once; per tile and K-step only the start
      // address field (bytes >> 4, low bits) moves.
      const uint64_t qd = smem_desc_sw128(sbase + C::kQOff + qsel * C::kQBytes, 16, 1024);
      const uint64_t kd0 = smem_desc_sw128(sbase + C::kKOff, 16, 1024);
      const uint64_t vd0 = smem_desc_sw128(sbase + C::kVOff, C::kBlk, 1024);
      const uint32_t tS = tmem + C::kSCol + l * 128;  // + 64 b: S / P buffer b
      const uint32_t tO = tmem + C::kOCol + l * D;
      auto wait_w = [&](uint32_t bar, uint32_t par) -> bool {
        const bool w = mbar_wait_spin(bar, par, abort_flag, p.err);
        return __all_sync(0xffffffffu, w);
      };
      // QK(j) into S buffer j & 1; the buffer is free once PV(j - 2), which
      // read P(j - 2) from it, has completed.
      auto qk = [&](int j) -> bool {
        const int g = item_of(l, j);
        const int s = g % KS;
        if (!wait_w(b_kfull(s), (g / KS) & 1)) return false;
        tc_fence_after();
        const uint64_t kd = kd0 + static_cast<uint64_t>(s * (C::kKVBytes >> 4));
        if (leader) {
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t qo = ((kk >> 2) * C::kQBlk + (kk & 3) * 32) >> 4;
            const uint32_t ko = ((kk >> 2) * C::kBlk + (kk & 3) * 32) >> 4;
            umma_ss(tS + (j & 1) * 64, qd + qo, kd + ko, idesc_qk, kk > 0 ? 1u : 0u);
          }
          umma_commit(b_sfull(l, j & 1));
          umma_commit(b_kempty(s));
        }
        __syncwarp();
        return true;
      };
      bool ok = wait_w(b_qfull, 0) && qk(0) && (nl < 2 || qk(1));
      for (int jp = 0; ok && jp < nl; ++jp) {
        const int g = item_of(l, jp);
        const int s = g % VS;
        const int b = jp & 1;
        if (!wait_w(b_pfull(l, b), (jp >> 1) & 1)) { ok = false; break; }
        if (!wait_w(b_vfull(s), (g / VS) & 1)) { ok = false; break; }
        tc_fence_after();
        const uint64_t vd = vd0 + static_cast<uint64_t>(s * (C::kKVBytes >> 4));
        if (leader) {
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk)
            umma_ts(tO, tS + b * 64 + kk * 8, vd + static_cast<uint64_t>(kk * (2048 >> 4)),
                    idesc_pv, (jp > 0 || kk > 0) ? 1u : 0u);
          umma_commit(b_pvdone(l, b));
          umma_commit(b_vempty(s));
        }
        __syncwarp();
        if (jp + 2 < nl) {
          if (!wait_w(b_pvdone(l, b), (jp >> 1) & 1)) { ok = false; break; }
          if (!qk(jp + 2)) { ok = false; break; }
        }
      }
      if (!ok) {
        // Drain: wait for every MMA the leader issued before TMEM is released.
        if (leader) umma_commit(b_drain(l));
        __syncwarp();
        mbar_wait(b_drain(l), 0, nullptr, p.err, 100000000ull);
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ softmax lanes
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));
    const int ln = (warp - 4) >> 2;  // 0 for warps 4..7, 1 for warps 8..11
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane_id;
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(q4 * 32) << 16);
    const uint32_t tS = t_lane + C::kSCol + ln * 128;  // + 64 (j & 1)
    const uint32_t tO = t_lane + C::kOCol + ln * D;
    const int my_n = ln == 0 ? n0 : n1;
    const int tile0 = kb + ((split && ln == 1) ? n0 : 0);
    const int qi = (alt ? qt0 : qt0 + ln) * BM + row;
    const int ohead = xh ? head + ln : head;  // the head this lane's rows belong to
    const float sl = p.scale_log2;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    auto wait_all = [&](uint32_t bar, uint32_t par) -> bool {
      bool w = mbar_wait(bar, par, abort_flag, p.err);
      return __shfl_sync(0xffffffffu, w ? 1 : 0, 0) != 0;
    };
    const uint64_t sl2 = f2_packf(sl, sl);
    for (int j = 0; j < my_n; ++j) {
      if (!wait_all(b_sfull(ln, j & 1), (j >> 1) & 1)) { ok = false; break; }
      tc_fence_after();
      const uint32_t tSj = tS + (j & 1) * 64;
      uint32_t sr[BN];
      TM_TMEM_LD32(tSj + 0, (sr + 0));
      TM_TMEM_LD32(tSj + 32, (sr + 32));
      tmem_wait_ld();

      const int valid = tl[tile0 + j].y;
      if (valid < BN) {
#pragma unroll
        for (int c = 0; c < BN; ++c)
          if (c >= valid) sr[c] = __float_as_uint(-INFINITY);
      }
      float mxa = fmax3f(__uint_as_float(sr[0]), __uint_as_float(sr[1]), __uint_as_float(sr[2]));
      float mxb = fmax3f(__uint_as_float(sr[3]), __uint_as_float(sr[4]), __uint_as_float(sr[5]));
      float mxc = fmax3f(__uint_as_float(sr[6]), __uint_as_float(sr[7]), __uint_as_float(sr[8]));
      float mxd = fmax3f(__uint_as_float(sr[9]), __uint_as_float(sr[10]), __uint_as_float(sr[11]));
#pragma unroll
      for (int c = 12; c < 60; c += 8) {
        mxa = fmax3f(mxa, __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]));
        mxb = fmax3f(mxb, __uint_as_float(sr[c + 2]), __uint_as_float(sr[c + 3]));
        mxc = fmax3f(mxc, __uint_as_float(sr[c + 4]), __uint_as_float(sr[c + 5]));
        mxd = fmax3f(mxd, __uint_as_float(sr[c + 6]), __uint_as_float(sr[c + 7]));
      }
      mxa = fmax3f(mxa, __uint_as_float(sr[60]), __uint_as_float(sr[61]));
      mxb = fmax3f(mxb, __uint_as_float(sr[62]), __uint_as_float(sr[63]));
      const float mx = fmaxf(fmaxf(mxa, mxb), fmaxf(mxc, mxd));
      const float mx_s = mx * sl;
      // Lazy rescale: the reference max moves only when the row max grows by
      // more than 2^8; O and the running sum are then scaled by alpha.
      bool need = false;
      float alpha = 1.0f;
      if (j == 0) {
        m_run = mx_s;
      } else if (mx_s > m_run + 8.0f) {
        need = true;
        alpha = ex2_approx(m_run - mx_s);
        m_run = mx_s;
      }
      const uint64_t nm2 = f2_packf(-m_run, -m_run);
      uint64_t acc[4] = {0, 0, 0, 0};
      uint32_t pk[BN / 2];
#pragma unroll
      for (int c = 0; c < BN; c += 2) {
        float x0, x1, p0, p1;
        f2_unpack(f2_fma(f2_pack(sr[c], sr[c + 1]), sl2, nm2), x0, x1);
        if (((c >> 1) & 3) < kEmulPairs) {
          exp2_poly2(x0, x1, p0, p1);
        } else {
          p0 = ex2_approx(x0);
          p1 = ex2_approx(x1);
        }
        acc[(c >> 1) & 3] = f2_add(acc[(c >> 1) & 3], f2_packf(p0, p1));
        pk[c >> 1] = pack_bf16x2(p0, p1);
      }
      float a0, a1, a2, a3;
      f2_unpack(f2_add(acc[0], acc[1]), a0, a1);
      f2_unpack(f2_add(acc[2], acc[3]), a2, a3);
      l_run = l_run * alpha + ((a0 + a1) + (a2 + a3));
      if (__any_sync(0xffffffffu, need)) {
        // O_l must hold PV(j - 1) before it is rescaled; PV(j) is issued only
        // after this thread's p_full arrival below.
        if (!wait_all(b_pvdone(ln, (j - 1) & 1), ((j - 1) >> 1) & 1)) { ok = false; break; }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < D / 16; ++c) {
          uint32_t o[16];
          TM_TMEM_LD16(tO + c * 16, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          TM_TMEM_ST16(tO + c * 16, o);
        }
      }
      // P(j) over the first half of its own S buffer (S(j) is in registers;
      // the next MMA to write this buffer waits for PV(j)).
      TM_TMEM_ST32(tSj, pk);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(b_pfull(ln, j & 1));
    }
    // the final PV of this lane
    const bool fin =
        ok && my_n > 0 && wait_all(b_pvdone(ln, (my_n - 1) & 1), ((my_n - 1) >> 1) & 1);
    if (split && ln == 1) {
      m1_smem[row] = fin ? m_run : -INFINITY;
      l1_smem[row] = fin ? l_run : 0.f;
    }
    named_bar_sync(1, 256);
    const bool writer = split ? (ln == 0) : true;
    bool ok1 = true;
    if (split && ln == 0 && fin)
      ok1 = (n1 == 0) || wait_all(b_pvdone(1, (n1 - 1) & 1), ((n1 - 1) >> 1) & 1);
    if (writer && fin && ok1) {
      tc_fence_after();
      float s0 = 1.0f / l_run, s1 = 0.f;
      const bool merge = split && n1 > 0;
      if (merge) {
        const float m1 = m1_smem[row], l1 = l1_smem[row];
        const float m = fmaxf(m_run, m1);
        const float c0 = ex2_approx(m_run - m);
        const float c1 = l1 > 0.f ? ex2_approx(m1 - m) : 0.f;
        const float inv = 1.0f / (l_run * c0 + l1 * c1);
        s0 = c0 * inv;
        s1 = c1 * inv;
      }
      const uint32_t tO1 = t_lane + C::kOCol + D;
      if (p.part_o) {
        // Normalised partial output of this key range, and its (max, sum).
        // The TMEM loads are warp-collective: every lane runs them, rows past
        // Lq only skip the stores.
        const bool live = qi < p.Lq;
        const int64_t idx =
            ((static_cast<int64_t>(sidx) * gridDim.z + batch) * p.Lq + qi) * gridDim.x + head;
        float m_tot = m_run, l_tot = l_run;
        if (merge) {
          const float m1 = m1_smem[row], l1 = l1_smem[row];
          m_tot = fmaxf(m_run, m1);
          l_tot = l_run * ex2_approx(m_run - m_tot) + (l1 > 0.f ? l1 * ex2_approx(m1 - m_tot) : 0.f);
        }
        if (live) p.part_ml[idx] = make_float2(m_tot, l_tot);
        float* prow = p.part_o + idx * D;
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32], o1[32];
          TM_TMEM_LD32(tO + c * 32, o);
          if (merge) {
            TM_TMEM_LD32(tO1 + c * 32, o1);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) o1[i] = 0u;
          }
          tmem_wait_ld();
          if (live) {
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
              float4 v;
              v.x = __uint_as_float(o[i]) * s0 + __uint_as_float(o1[i]) * s1;
              v.y = __uint_as_float(o[i + 1]) * s0 + __uint_as_float(o1[i + 1]) * s1;
              v.z = __uint_as_float(o[i + 2]) * s0 + __uint_as_float(o1[i + 2]) * s1;
              v.w = __uint_as_float(o[i + 3]) * s0 + __uint_as_float(o1[i + 3]) * s1;
              *reinterpret_cast<float4*>(prow + c * 32 + i) = v;
            }
          }
        }
      } else {
      if (qi < p.Lq) {
        const float g = gate_of(p.gate, p.gate_bs, p.gate_rs, batch, qi, ohead);
        s0 *= g;
        s1 *= g;
      }
      if (!p.stage_out) {
        // every row stays on this GPU: each thread stores its own row
        __nv_bfloat16* orow = out_row(p.out, p.out_bs, p.out_rs, p.rows_per_rank, p.head_base,
                                      p.out_delta, batch, qi, ohead, D);
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32], o1[32];
          TM_TMEM_LD32(tO + c * 32, o);
          if (merge) {
            TM_TMEM_LD32(tO1 + c * 32, o1);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) o1[i] = 0u;
          }
          tmem_wait_ld();
          if (qi < p.Lq) {
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              float f[8];
#pragma unroll
              for (int k = 0; k < 8; ++k)
                f[k] = __uint_as_float(o[i + k]) * s0 + __uint_as_float(o1[i + k]) * s1;
              const uint4 v = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]),
                                         pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
              *reinterpret_cast<uint4*>(orow + c * 32 + i) = v;
            }
          }
        }
      } else {
      // Rows go to other GPUs: the warp's 32 rows x D bf16 go through a free
      // Q buffer (split CTAs never load buffer 1; in a pair CTA this lane's
      // own buffer, whose last MMA has completed), in 16-byte pieces
      // XOR-swizzled by row, so that each warp store covers whole rows
      // (32 / (D / 8) rows of 2 D contiguous bytes) instead of 32 scattered
      // pieces, and crosses NVLink in full lines.
      constexpr int kPieces = D / 8;
      uint4* stg = reinterpret_cast<uint4*>(smem + C::kQOff + (split ? 1 : ln) * C::kQBytes) +
                   q4 * 32 * kPieces;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32], o1[32];
        TM_TMEM_LD32(tO + c * 32, o);
        if (merge) {
          TM_TMEM_LD32(tO1 + c * 32, o1);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o1[i] = 0u;
        }
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          float f[8];
#pragma unroll
          for (int k = 0; k < 8; ++k)
            f[k] = __uint_as_float(o[i + k]) * s0 + __uint_as_float(o1[i + k]) * s1;
          const int pc = c * 4 + (i >> 3);
          stg[lane_id * kPieces + (pc ^ (lane_id & (kPieces - 1)))] =
              make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]),
                         pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
        }
      }
      __syncwarp();
      constexpr int kRowsPer = 32 / kPieces;
      const int qw = qi - lane_id;  // the warp's first row
      const int pc = lane_id % kPieces;
#pragma unroll 4
      for (int i = 0; i < 32 / kRowsPer; ++i) {
        const int rr = i * kRowsPer + lane_id / kPieces;
        if (qw + rr < p.Lq) {
          __nv_bfloat16* orow = out_row(p.out, p.out_bs, p.out_rs, p.rows_per_rank, p.head_base,
                                        p.out_delta, batch, qw + rr, ohead, D);
          *reinterpret_cast<uint4*>(orow + pc * 8) =
              stg[rr * kPieces + (pc ^ (rr & (kPieces - 1)))];
        }
      }
      }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// Merge of partial outputs: one warp per (batch, query row, head); out =
// sum_s w_s O_s / sum_s w_s with w_s = l_s 2^(m_s - max_s m_s), O_s a key
// range's normalised output.  The partials come in n_groups groups of kvs
// (group g at byte offset g * group_bytes from part_o / part_ml: one group per
// GPU of a gathered exchange), merged in group-major order, so every GPU that
// merges the same gathered bytes stores the same bits.
struct OutPlace {
  __nv_bfloat16* out;
  int64_t out_bs, out_rs;
  int rows_per_rank, head_base;
  int64_t delta[8];
  const __nv_bfloat16* gate;
  int64_t gate_bs, gate_rs;
};

template <int D>
__global__ void __launch_bounds__(256) combine_kernel(const float* __restrict__ part_o,
                                                      const float2* __restrict__ part_ml, int kvs,
                                                      int n_groups, int64_t group_bytes,
                                                      int B, int Lq, int H,
                                                      const __grid_constant__ OutPlace op) {
  constexpr int kPer = D / 32;  // columns per lane
  const int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t total = static_cast<int64_t>(B) * Lq * H;
  if (w >= total) return;
  const int h = static_cast<int>(w % H);
  const int qi = static_cast<int>((w / H) % Lq);
  const int b = static_cast<int>(w / (static_cast<int64_t>(H) * Lq));
  const int np = n_groups * kvs;
  auto ml_of = [&](int i) {
    const int g = i / kvs, s = i - g * kvs;
    return reinterpret_cast<const float2*>(reinterpret_cast<const char*>(part_ml) +
                                           g * group_bytes)[s * total + w];
  };
  float mmax = -INFINITY;
  for (int i = 0; i < np; ++i) mmax = fmaxf(mmax, ml_of(i).x);
  float acc[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) acc[i] = 0.f;
  float den = 0.f;
  for (int i = 0; i < np; ++i) {
    const float2 ml = ml_of(i);
    // a group without keys has (max, sum) = (-inf, 0): weight 0
    const float wgt = ml.y > 0.f ? ml.y * exp2f(ml.x - mmax) : 0.f;
    den += wgt;
    const int g = i / kvs, s = i - g * kvs;
    const float* src = reinterpret_cast<const float*>(reinterpret_cast<const char*>(part_o) +
                                                      g * group_bytes) +
                       (s * total + w) * D + lane * kPer;
    if constexpr (kPer == 4) {
      const float4 v = *reinterpret_cast<const float4*>(src);
      acc[0] += wgt * v.x;
      acc[1] += wgt * v.y;
      acc[2] += wgt * v.z;
      acc[3] += wgt * v.w;
    } else {
      const float2 v = *reinterpret_cast<const float2*>(src);
      acc[0] += wgt * v.x;
      acc[1] += wgt * v.y;
    }
  }
  const float inv = gate_of(op.gate, op.gate_bs, op.gate_rs, b, qi, h) / den;
  __nv_bfloat16* dst = out_row(op.out, op.out_bs, op.out_rs, op.rows_per_rank, op.head_base,
                               op.delta, b, qi, h, D) + lane * kPer;
  if constexpr (kPer == 4) {
    *reinterpret_cast<uint2*>(dst) =
        make_uint2(pack_bf16x2(acc[0] * inv, acc[1] * inv), pack_bf16x2(acc[2] * inv, acc[3] * inv));
  } else {
    *reinterpret_cast<uint32_t*>(dst) = pack_bf16x2(acc[0] * inv, acc[1] * inv);
  }
}

// Encode a [B, rows, H, D] bf16 tensor (heads contiguous) as a 4-D TMA map
// with a {64, 1, box_rows, 1} box and 128-byte swizzle; rows past `rows` read
// as zero.
static int make_map(CUtensorMap* m, const void* base, int64_t rows, int B, int H, int D,
                    int64_t batch_stride, int64_t row_stride, int box_rows, const char* what) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return set_error(TM_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (B == 1) batch_stride = rows * row_stride;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(H),
                        static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(B)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(D) * 2, static_cast<cuuint64_t>(row_stride) * 2,
                           static_cast<cuuint64_t>(batch_stride) * 2};
  cuuint32_t box[4] = {64, 1, static_cast<cuuint32_t>(box_rows), 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(TM_ERR_CUDA, "tensor map for %s rejected (CUresult %d)", what, (int)r);
  return TM_OK;
}

template <int D>
static int launch(Params& prm, int B, int Lq, int H, cudaStream_t stream) {
  using C = Cfg<D>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    int st = check_cuda(cudaFuncSetAttribute(attn_fwd_kernel<D>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             C::kSmemAlloc),
                        "attention: set smem attribute");
    if (st) return st;
    configured[dev] = true;
  }
  // mode 0: pair CTAs (two query tiles of a head each), then the odd tile's
  // split CTA, head-minor so that every head's pair CTAs launch before any
  // split CTA.  mode 2: the same grid; the odd tiles of heads h and h + 1 go
  // to head h's CTA (head h + 1's returns at once).  mode 1: one CTA per
  // (query tile, key range).
  const int nq = (Lq + BM - 1) / BM;
  dim3 grid(H, prm.mode != 1 ? nq / 2 + (nq & 1) : nq * prm.kv_splits, B);
  attn_fwd_kernel<D><<<grid, kThreads, C::kSmemAlloc, stream>>>(prm);
  int st = check_cuda(cudaGetLastError(), "attention: launch");
  if (st || prm.kv_splits <= 1 || prm.partial_only) return st;
  const int64_t warps = static_cast<int64_t>(B) * Lq * H;
  OutPlace op;
  op.out = prm.out;
  op.out_bs = prm.out_bs;
  op.out_rs = prm.out_rs;
  op.rows_per_rank = prm.rows_per_rank;
  op.head_base = prm.head_base;
  for (int i = 0; i < 8; ++i) op.delta[i] = prm.out_delta[i];
  op.gate = prm.gate;
  op.gate_bs = prm.gate_bs;
  op.gate_rs = prm.gate_rs;
  combine_kernel<D><<<static_cast<unsigned>((warps + 7) / 8), 256, 0, stream>>>(
      prm.part_o, prm.part_ml, prm.kv_splits, 1, 0, B, Lq, H, op);
  return check_cuda(cudaGetLastError(), "attention: combine launch");
}

// Work partition.  Costs are in units of one query tile against all visible
// keys on one SM; CTAs start in grid order on the first free SM.
struct Plan {
  int mode;
  int kv_splits;
};

// Partial outputs of kvs key ranges: [kvs][B][Lq][H][D] fp32, then (at the
// next multiple of 256 bytes from the start, so that the layout does not
// depend on the buffer's address) [kvs][B][Lq][H] (max, sum).
static int64_t partial_ml_offset(int64_t rows, int D) {
  return (rows * D * 4 + 255) / 256 * 256;
}

static int64_t partial_bytes(int kvs, int B, int Lq, int H, int D) {
  const int64_t rows = static_cast<int64_t>(kvs) * B * Lq * H;
  return rows * D * 4 + rows * 8 + 256;
}

static int64_t split_ws_bytes(int kvs, int B, int Lq, int H, int D) {
  return kvs <= 1 ? 0 : partial_bytes(kvs, B, Lq, H, D);
}

static int sm_count() {
  static int counts[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev < 0 || dev >= 64) return 148;
  if (counts[dev] == 0) {
    int c = 0;
    if (cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || c <= 0)
      c = 148;
    counts[dev] = c;
  }
  return counts[dev];
}

// One unit = one query tile against all visible keys with both softmax lanes
// splitting the key tiles (n_tiles / 2 lane steps).  Every CTA also pays a
// fixed cost (TMEM allocation, barrier setup, the Q load, the epilogue)
// worth kFixedLaneSteps key-tile steps of one lane, so splitting a tiny query
// chunk into many short CTAs (V2A's 25 audio queries) stops paying off once
// the splits fill one wave.
constexpr double kFixedLaneSteps = 6.0;

static Plan make_plan(int B, int Lq, int H, int D, int n_tiles, int64_t ws_bytes) {
  const int sms = sm_count();
  const int64_t nq = (Lq + BM - 1) / BM;
  const int64_t heads = static_cast<int64_t>(H) * B;
  const int64_t big = heads * (nq / 2), small = heads * (nq & 1);
  const double c0 = kFixedLaneSteps / std::max(1.0, 0.5 * n_tiles);  // in units
  const auto waves = [sms](int64_t ctas) { return static_cast<double>((ctas + sms - 1) / sms); };
  // pair mode: 2-unit CTAs, then 1-unit CTAs
  const double cost_pair = std::max(waves(big) * (2.0 + c0),
                                    std::ceil(static_cast<double>(2 * big + small) / sms) +
                                        c0 * waves(big + small));
  Plan best{0, 1};
  double best_cost = cost_pair;
  // mode 2: with an odd tile count, the odd tiles of two heads share one
  // 2-unit CTA (each lane its own head), so every CTA carries 2 units: one
  // wave where pair mode spills the odd tiles' CTAs into a second one.
  if ((nq & 1) && H >= 2) {
    const int64_t ctas = static_cast<int64_t>(B) * (H * (nq / 2) + (H + 1) / 2);
    const double cost2 = waves(ctas) * (2.0 + c0);
    if (cost2 < best_cost - 1e-9) {
      best_cost = cost2;
      best = Plan{2, 1};
    }
  }
  const int s_max = std::max(1, std::min(32, n_tiles / 2));
  for (int s = 1; s <= s_max; ++s) {
    if (s > 1 && split_ws_bytes(s, B, Lq, H, D) > ws_bytes) break;
    const int64_t ctas = heads * nq * s;
    // the merge pass of s > 1 costs a little: require a clear gain
    const double cost = waves(ctas) * (1.0 / s + c0) * (s > 1 ? 1.08 : 1.0);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = Plan{1, s};
    }
  }
  return best;
}

// Key ranges per query tile for an export (every CTA a split CTA).
static int best_splits(int B, int Lq, int H, int n_tiles) {
  const int sms = sm_count();
  const int64_t ctas1 = static_cast<int64_t>(H) * B * ((Lq + BM - 1) / BM);
  const double c0 = kFixedLaneSteps / std::max(1.0, 0.5 * n_tiles);
  const int s_max = std::max(1, std::min(32, n_tiles / 2));
  int best = 1;
  double best_cost = 1e300;
  for (int s = 1; s <= s_max; ++s) {
    const double cost = static_cast<double>((ctas1 * s + sms - 1) / sms) * (1.0 / s + c0);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = s;
    }
  }
  return best;
}

}  // namespace attn
}  // namespace tmb

using namespace tmb;

// Key-tile list of a span list: (source << 30 | first row, valid rows), BN keys per tile.
static int build_tiles(const tm_kv_span* spans, int n_spans, int64_t cache_rows, int64_t new_rows,
                       int2* tiles, int* n_tiles, bool use_src[2]) {
  using namespace tmb::attn;
  int nt = 0;
  int64_t total = 0;
  for (int i = 0; i < n_spans; ++i) {
    const tm_kv_span& s = spans[i];
    if (s.source != TM_KV_SOURCE_CACHE && s.source != TM_KV_SOURCE_NEW)
      return set_error(TM_ERR_INVALID_ARGUMENT, "attention: span %d has source %d", i, s.source);
    const int64_t lim = s.source == TM_KV_SOURCE_CACHE ? cache_rows : new_rows;
    if (s.rows < 0 || s.row_start < 0 || (int64_t)s.row_start + s.rows > lim)
      return set_error(TM_ERR_INVALID_ARGUMENT,
                       "attention: span %d [%d, +%d) outside source of %lld rows", i, s.row_start,
                       s.rows, (long long)lim);
    if (s.rows == 0) continue;
    use_src[s.source] = true;
    for (int off = 0; off < s.rows; off += BN) {
      if (nt >= kMaxTiles)
        return set_error(TM_ERR_INVALID_ARGUMENT, "attention: more than %d visible keys",
                         kMaxTiles * BN);
      tiles[nt].x = (s.source << 30) | (s.row_start + off);
      tiles[nt].y = (s.rows - off) < BN ? (s.rows - off) : BN;
      ++nt;
    }
    total += s.rows;
  }
  if (total == 0) return set_error(TM_ERR_INVALID_ARGUMENT, "attention: no visible keys");
  *n_tiles = nt;
  return TM_OK;
}

static tm_attention_ext ext_ws(void* ws, int64_t bytes, const void* tiles = nullptr) {
  tm_attention_ext e{};
  e.workspace = ws;
  e.workspace_bytes = bytes;
  e.device_tiles = tiles;
  return e;
}

static int attention_impl(const void* q, int64_t q_batch_stride, int64_t q_row_stride,
                          const void* k_cache, const void* v_cache, int64_t cache_batch_stride,
                          int64_t cache_row_stride, int64_t cache_rows, const void* k_new,
                          const void* v_new, int64_t new_batch_stride, int64_t new_row_stride,
                          int64_t new_rows, const tm_kv_span* spans, int n_spans, void* out,
                          int64_t out_batch_stride, int64_t out_row_stride, int B, int Lq, int H,
                          int D, float scale, const tm_attention_ext& ext, void* stream) {
  using namespace tmb::attn;
  void* workspace = ext.workspace;
  const int64_t workspace_bytes = ext.workspace_bytes;
  const void* device_tiles = ext.device_tiles;
  if (D != 64 && D != 128) return set_error(TM_ERR_UNSUPPORTED, "attention: head dim %d", D);
  if (B < 1 || Lq < 1 || H < 1 || B > 65535 || H > 65535 || (Lq + 255) / 256 > 65535)
    return set_error(TM_ERR_INVALID_ARGUMENT, "attention: B=%d Lq=%d H=%d", B, Lq, H);
  const bool export_parts = ext.parts != nullptr;
  if (export_parts) {
    // partial results only: `out` and everything about its placement go unused
    if (ext.part_splits < 1 || ext.parts_bytes < partial_bytes(ext.part_splits, B, Lq, H, D))
      return set_error(TM_ERR_INVALID_ARGUMENT, "attention: %d key ranges need %lld bytes of parts",
                       ext.part_splits,
                       (long long)partial_bytes(std::max(1, ext.part_splits), B, Lq, H, D));
    if (!aligned16(ext.parts))
      return set_error(TM_ERR_ALIGNMENT, "attention: parts not 16-byte aligned");
    out = ext.parts;
    out_batch_stride = 0;
    out_row_stride = static_cast<int64_t>(H) * D;
  }
  if (!q || !out || !spans || n_spans < 1)
    return set_error(TM_ERR_INVALID_ARGUMENT, "attention: null pointer or no spans");
  if (!aligned16(q) || !aligned16(out))
    return set_error(TM_ERR_ALIGNMENT, "attention: q/out not 16-byte aligned");
  const int64_t strides[6] = {q_batch_stride, q_row_stride, out_batch_stride, out_row_stride,
                              cache_row_stride, new_row_stride};
  for (int i = 0; i < 6; ++i)
    if (strides[i] < 0 || (strides[i] & 7))
      return set_error(TM_ERR_ALIGNMENT, "attention: stride %lld not a multiple of 8 elements",
                       (long long)strides[i]);
  if ((B > 1) && ((cache_batch_stride & 7) || (new_batch_stride & 7)))
    return set_error(TM_ERR_ALIGNMENT, "attention: batch stride not a multiple of 8 elements");
  if (q_row_stride < (int64_t)H * D || out_row_stride < (int64_t)H * D)
    return set_error(TM_ERR_INVALID_ARGUMENT, "attention: row stride smaller than H*D");

  Params prm;
  memset(&prm, 0, sizeof(prm));
  bool use_src[2] = {false, false};
  int nt = 0;
  int st0 = build_tiles(spans, n_spans, cache_rows, new_rows, prm.tiles, &nt, use_src);
  if (st0) return st0;
  if (device_tiles) {
    // the device table is rewritten between graph replays: map every given source
    if (!aligned16(device_tiles))
      return set_error(TM_ERR_ALIGNMENT, "attention: device tile table not 16-byte aligned");
    use_src[0] = use_src[0] || (k_cache && v_cache);
    use_src[1] = use_src[1] || (k_new && v_new);
    prm.tiles_dev = static_cast<const int2*>(device_tiles);
  }
  const void* kp[2] = {k_cache, k_new};
  const void* vp[2] = {v_cache, v_new};
  const int64_t rows_of[2] = {cache_rows, new_rows};
  const int64_t bs_of[2] = {cache_batch_stride, new_batch_stride};
  const int64_t rs_of[2] = {cache_row_stride, new_row_stride};
  for (int s = 0; s < 2; ++s) {
    if (!use_src[s]) continue;
    if (!kp[s] || !vp[s])
      return set_error(TM_ERR_INVALID_ARGUMENT, "attention: source %d referenced but null", s);
    if (!aligned16(kp[s]) || !aligned16(vp[s]))
      return set_error(TM_ERR_ALIGNMENT, "attention: source %d not 16-byte aligned", s);
    if (rs_of[s] < (int64_t)H * D)
      return set_error(TM_ERR_INVALID_ARGUMENT, "attention: source %d row stride < H*D", s);
  }
  int st = TM_OK;
  for (int s = 0; s < 2; ++s) {
    const int src = use_src[s] ? s : (use_src[0] ? 0 : 1);  // unused slot: copy a valid map
    st = make_map(&prm.tm_k[s], kp[src], rows_of[src], B, H, D, bs_of[src], rs_of[src], BN, "k");
    if (st) return st;
    st = make_map(&prm.tm_v[s], vp[src], rows_of[src], B, H, D, bs_of[src], rs_of[src], BN, "v");
    if (st) return st;
  }
  st = make_map(&prm.tm_q, q, Lq, B, H, D, q_batch_stride, q_row_stride, BM, "q");
  if (st) return st;
  prm.n_tiles = nt;
  prm.n_qtiles = (Lq + BM - 1) / BM;
  prm.Lq = Lq;
  prm.out = static_cast<__nv_bfloat16*>(out);
  prm.out_bs = (B == 1) ? 0 : out_batch_stride;
  prm.out_rs = out_row_stride;
  if (export_parts) {
    if (ext.part_splits > nt)
      return set_error(TM_ERR_INVALID_ARGUMENT, "attention: %d key ranges over %d key tiles",
                       ext.part_splits, nt);
    prm.rows_per_rank = Lq;
    prm.mode = 1;
    prm.kv_splits = ext.part_splits;
    prm.partial_only = 1;
    const int64_t rows = static_cast<int64_t>(ext.part_splits) * B * Lq * H;
    prm.part_o = static_cast<float*>(ext.parts);
    prm.part_ml = reinterpret_cast<float2*>(reinterpret_cast<char*>(prm.part_o) +
                                            partial_ml_offset(rows, D));
    const double sc = (scale > 0.f) ? (double)scale : 1.0 / std::sqrt((double)D);
    prm.scale_log2 = static_cast<float>(sc * 1.4426950408889634);
    prm.err = device_error_flag();
    if (!prm.err) return set_error(TM_ERR_CUDA, "attention: device error flag unavailable");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    return D == 128 ? launch<128>(prm, B, Lq, H, s) : launch<64>(prm, B, Lq, H, s);
  }
  prm.rows_per_rank = ext.rows_per_rank > 0 ? ext.rows_per_rank : Lq;
  prm.head_base = ext.head_base;
  if (ext.rows_per_rank < 0 || ext.head_base < 0 ||
      (ext.rows_per_rank > 0 && (Lq + ext.rows_per_rank - 1) / ext.rows_per_rank > 8))
    return set_error(TM_ERR_INVALID_ARGUMENT, "attention: output placement rows %d head %d",
                     ext.rows_per_rank, ext.head_base);
  if (out_row_stride < static_cast<int64_t>(ext.head_base + H) * D)
    return set_error(TM_ERR_INVALID_ARGUMENT, "attention: output row stride below head_base+H");
  for (int i = 0; i < 8; ++i) {
    if (ext.out_delta[i] & 15)
      return set_error(TM_ERR_ALIGNMENT, "attention: output offset %d not 16-byte aligned", i);
    prm.out_delta[i] = ext.out_delta[i];
    if (ext.out_delta[i] != 0) prm.stage_out = 1;
  }
  if (ext.gate_logits) {
    if (ext.gate_row_stride < H || ext.gate_batch_stride < 0)
      return set_error(TM_ERR_INVALID_ARGUMENT, "attention: gate row stride %lld < H",
                       (long long)ext.gate_row_stride);
    prm.gate = static_cast<const __nv_bfloat16*>(ext.gate_logits);
    prm.gate_bs = (B == 1) ? 0 : ext.gate_batch_stride;
    prm.gate_rs = ext.gate_row_stride;
  }
  const double sc = (scale > 0.f) ? (double)scale : 1.0 / std::sqrt((double)D);
  prm.scale_log2 = static_cast<float>(sc * 1.4426950408889634);
  prm.err = device_error_flag();
  if (!prm.err) return set_error(TM_ERR_CUDA, "attention: device error flag unavailable");
  if (workspace_bytes < 0 || (workspace_bytes > 0 && !workspace))
    return set_error(TM_ERR_INVALID_ARGUMENT, "attention: bad workspace");
  if (workspace && !aligned16(workspace))
    return set_error(TM_ERR_ALIGNMENT, "attention: workspace not 16-byte aligned");
  const Plan plan = make_plan(B, Lq, H, D, nt, workspace ? workspace_bytes : 0);
  prm.mode = plan.mode;
  prm.kv_splits = plan.kv_splits;
  if (plan.kv_splits > 1) {
    const int64_t rows = static_cast<int64_t>(plan.kv_splits) * B * Lq * H;
    prm.part_o = static_cast<float*>(workspace);
    prm.part_ml = reinterpret_cast<float2*>(reinterpret_cast<char*>(prm.part_o) +
                                            partial_ml_offset(rows, D));
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return D == 128 ? launch<128>(prm, B, Lq, H, s) : launch<64>(prm, B, Lq, H, s);
}

extern "C" int tm_attention_fwd(const void* q, int64_t q_batch_stride, int64_t q_row_stride,
                                const void* k_cache, const void* v_cache,
                                int64_t cache_batch_stride, int64_t cache_row_stride,
                                int64_t cache_rows, const void* k_new, const void* v_new,
                                int64_t new_batch_stride, int64_t new_row_stride, int64_t new_rows,
                                const tm_kv_span* spans, int n_spans, void* out,
                                int64_t out_batch_stride, int64_t out_row_stride, int B, int Lq,
                                int H, int D, float scale, void* stream) {
  return attention_impl(q, q_batch_stride, q_row_stride, k_cache, v_cache, cache_batch_stride,
                        cache_row_stride, cache_rows, k_new, v_new, new_batch_stride,
                        new_row_stride, new_rows, spans, n_spans, out, out_batch_stride,
                        out_row_stride, B, Lq, H, D, scale, tm_attention_ext{}, stream);
}

extern "C" int tm_attention_fwd_ws(const void* q, int64_t q_batch_stride, int64_t q_row_stride,
                                   const void* k_cache, const void* v_cache,
                                   int64_t cache_batch_stride, int64_t cache_row_stride,
                                   int64_t cache_rows, const void* k_new, const void* v_new,
                                   int64_t new_batch_stride, int64_t new_row_stride,
                                   int64_t new_rows, const tm_kv_span* spans, int n_spans,
                                   void* out, int64_t out_batch_stride, int64_t out_row_stride,
                                   int B, int Lq, int H, int D, float scale, void* workspace,
                                   int64_t workspace_bytes, void* stream) {
  return attention_impl(q, q_batch_stride, q_row_stride, k_cache, v_cache, cache_batch_stride,
                        cache_row_stride, cache_rows, k_new, v_new, new_batch_stride,
                        new_row_stride, new_rows, spans, n_spans, out, out_batch_stride,
                        out_row_stride, B, Lq, H, D, scale, ext_ws(workspace, workspace_bytes),
                        stream);
}

extern "C" int64_t tm_attention_workspace_bytes(int B, int Lq, int H, int D,
                                                int64_t visible_keys) {
  using namespace tmb::attn;
  if (B < 1 || Lq < 1 || H < 1 || (D != 64 && D != 128) || visible_keys < 1) return 0;
  const int64_t tiles = std::min<int64_t>((visible_keys + BN - 1) / BN, kMaxTiles);
  const Plan plan = make_plan(B, Lq, H, D, static_cast<int>(tiles), INT64_MAX);
  return split_ws_bytes(plan.kv_splits, B, Lq, H, D);
}

extern "C" int tm_attention_plan(int B, int Lq, int H, int D, int64_t visible_keys,
                                 int64_t workspace_bytes, int* mode, int* kv_splits, int* ctas) {
  using namespace tmb::attn;
  if (!mode || !kv_splits || !ctas)
    return set_error(TM_ERR_INVALID_ARGUMENT, "attention_plan: null output");
  if (B < 1 || Lq < 1 || H < 1 || visible_keys < 1 || workspace_bytes < 0)
    return set_error(TM_ERR_INVALID_ARGUMENT, "attention_plan: B=%d Lq=%d H=%d keys=%lld", B,
                     Lq, H, (long long)visible_keys);
  if (D != 64 && D != 128) return set_error(TM_ERR_UNSUPPORTED, "attention_plan: head dim %d", D);
  if ((visible_keys + BN - 1) / BN > kMaxTiles)
    return set_error(TM_ERR_INVALID_ARGUMENT, "attention_plan: more than %d visible keys",
                     kMaxTiles * BN);
  const int tiles = static_cast<int>((visible_keys + BN - 1) / BN);
  const Plan plan = make_plan(B, Lq, H, D, tiles, workspace_bytes);
  const int64_t nq = (Lq + BM - 1) / BM;
  int64_t n = 0;
  if (plan.mode == 1)
    n = static_cast<int64_t>(B) * H * nq * plan.kv_splits;
  else if (plan.mode == 2)
    n = static_cast<int64_t>(B) * (H * (nq / 2) + (H + 1) / 2);
  else
    n = static_cast<int64_t>(B) * H * (nq / 2 + (nq & 1));
  *mode = plan.mode;
  *kv_splits = plan.kv_splits;
  *ctas = static_cast<int>(std::min<int64_t>(n, 0x7fffffff));
  return TM_OK;
}

extern "C" int64_t tm_attention_partial_bytes(int B, int Lq, int H, int D, int splits) {
  using namespace tmb::attn;
  if (B < 1 || Lq < 1 || H < 1 || (D != 64 && D != 128) || splits < 1) return 0;
  return partial_bytes(splits, B, Lq, H, D);
}

extern "C" int tm_attention_partial_splits(int B, int Lq, int H, int D, int64_t visible_keys) {
  using namespace tmb::attn;
  if (B < 1 || Lq < 1 || H < 1 || (D != 64 && D != 128) || visible_keys < 1) return 1;
  const int tiles = static_cast<int>(std::min<int64_t>((visible_keys + BN - 1) / BN, kMaxTiles));
  return best_splits(B, Lq, H, tiles);
}

extern "C" int tm_attention_combine(const void* parts, int n_groups, int64_t group_bytes,
                                    int splits, int B, int Lq, int H, int D, void* out,
                                    int64_t out_batch_stride, int64_t out_row_stride,
                                    const void* gate_logits, int64_t gate_batch_stride,
                                    int64_t gate_row_stride, void* stream) {
  using namespace tmb::attn;
  if (D != 64 && D != 128) return set_error(TM_ERR_UNSUPPORTED, "combine: head dim %d", D);
  if (B < 1 || Lq < 1 || H < 1 || n_groups < 1 || splits < 1 || !parts || !out)
    return set_error(TM_ERR_INVALID_ARGUMENT, "combine: B=%d Lq=%d H=%d groups=%d splits=%d",
                     B, Lq, H, n_groups, splits);
  const int64_t need = partial_bytes(splits, B, Lq, H, D);
  if (n_groups > 1 && group_bytes < need)
    return set_error(TM_ERR_INVALID_ARGUMENT, "combine: group stride %lld below %lld bytes",
                     (long long)group_bytes, (long long)need);
  if (!aligned16(parts) || (group_bytes & 15))
    return set_error(TM_ERR_ALIGNMENT, "combine: parts or group stride not 16-byte aligned");
  if (!aligned16(out) || (out_row_stride & 7) || (out_batch_stride & 7) ||
      out_row_stride < static_cast<int64_t>(H) * D)
    return set_error(TM_ERR_ALIGNMENT, "combine: output alignment or strides");
  if (gate_logits && (gate_row_stride < H || gate_batch_stride < 0))
    return set_error(TM_ERR_INVALID_ARGUMENT, "combine: gate row stride %lld < H",
                     (long long)gate_row_stride);
  const int64_t rows = static_cast<int64_t>(splits) * B * Lq * H;
  const float* po = static_cast<const float*>(parts);
  const float2* ml = reinterpret_cast<const float2*>(reinterpret_cast<const char*>(po) +
                                                     partial_ml_offset(rows, D));
  OutPlace op;
  memset(&op, 0, sizeof(op));
  op.out = static_cast<__nv_bfloat16*>(out);
  op.out_bs = (B == 1) ? 0 : out_batch_stride;
  op.out_rs = out_row_stride;
  op.rows_per_rank = Lq;
  op.gate = static_cast<const __nv_bfloat16*>(gate_logits);
  op.gate_bs = (B == 1) ? 0 : gate_batch_stride;
  op.gate_rs = gate_row_stride;
  const int64_t warps = static_cast<int64_t>(B) * Lq * H;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const unsigned grid = static_cast<unsigned>((warps + 7) / 8);
  if (D == 128)
    combine_kernel<128><<<grid, 256, 0, s>>>(po, ml, splits,
                                             n_groups, group_bytes, B, Lq, H, op);
  else
    combine_kernel<64><<<grid, 256, 0, s>>>(po, ml, splits,
                                            n_groups, group_bytes, B, Lq, H, op);
  return check_cuda(cudaGetLastError(), "combine: launch");
}

extern "C" int tm_attention_tiles(const tm_kv_span* spans, int n_spans, int64_t cache_rows,
                                  int64_t new_rows, int32_t* tiles_out, int max_tiles,
                                  int* n_tiles) {
  using namespace tmb::attn;
  if (!spans || n_spans < 1 || !tiles_out || !n_tiles)
    return set_error(TM_ERR_INVALID_ARGUMENT, "attention tiles: null pointer or no spans");
  int2 tmp[kMaxTiles];
  bool use_src[2] = {false, false};
  int nt = 0;
  const int st = build_tiles(spans, n_spans, cache_rows, new_rows, tmp, &nt, use_src);
  if (st) return st;
  if (nt > max_tiles)
    return set_error(TM_ERR_INVALID_ARGUMENT, "attention tiles: %d tiles, room for %d", nt,
                     max_tiles);
  memcpy(tiles_out, tmp, sizeof(int2) * nt);
  *n_tiles = nt;
  return TM_OK;
}

extern "C" int tm_attention_fwd_dev_tiles(
    const void* q, int64_t q_batch_stride, int64_t q_row_stride, const void* k_cache,
    const void* v_cache, int64_t cache_batch_stride, int64_t cache_row_stride, int64_t cache_rows,
    const void* k_new, const void* v_new, int64_t new_batch_stride, int64_t new_row_stride,
    int64_t new_rows, const tm_kv_span* spans, int n_spans, const void* device_tiles, void* out,
    int64_t out_batch_stride, int64_t out_row_stride, int B, int Lq, int H, int D, float scale,
    void* workspace, int64_t workspace_bytes, void* stream) {
  if (!device_tiles)
    return set_error(TM_ERR_INVALID_ARGUMENT, "attention: null device tile table");
  return attention_impl(q, q_batch_stride, q_row_stride, k_cache, v_cache, cache_batch_stride,
                        cache_row_stride, cache_rows, k_new, v_new, new_batch_stride,
                        new_row_stride, new_rows, spans, n_spans, out, out_batch_stride,
                        out_row_stride, B, Lq, H, D, scale,
                        ext_ws(workspace, workspace_bytes, device_tiles), stream);
}

extern "C" int tm_attention_fwd_ext(const void* q, int64_t q_batch_stride, int64_t q_row_stride,
                                    const void* k_cache, const void* v_cache,
                                    int64_t cache_batch_stride, int64_t cache_row_stride,
                                    int64_t cache_rows, const void* k_new, const void* v_new,
                                    int64_t new_batch_stride, int64_t new_row_stride,
                                    int64_t new_rows, const tm_kv_span* spans, int n_spans,
                                    void* out, int64_t out_batch_stride, int64_t out_row_stride,
                                    int B, int Lq, int H, int D, float scale,
                                    const tm_attention_ext* ext, void* stream) {
  if (!ext) return set_error(TM_ERR_INVALID_ARGUMENT, "attention: null options");
  return attention_impl(q, q_batch_stride, q_row_stride, k_cache, v_cache, cache_batch_stride,
                        cache_row_stride, cache_rows, k_new, v_new, new_batch_stride,
                        new_row_stride, new_rows, spans, n_spans, out, out_batch_stride,
                        out_row_stride, B, Lq, H, D, scale, *ext, stream);
}

// ---------------------------------------------------------------------------
// Entry point for callers that cannot allocate device memory.  Its scratch
// (the key-range split's partial outputs) lives in a fixed array in this
// library's own device memory, so each GPU that loads the library holds
// kNoAllocScratchBytes of it until the process exits.  Host code must not pass
// the array's name to a kernel: on the host it only stands in for the symbol.
// The device address is looked up with cudaGetSymbolAddress once per device,
// with that device current, on the first call made on it.
namespace tmb {
namespace attn {

constexpr int64_t kNoAllocScratchBytes = int64_t(16) << 20;  // 16 MiB
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

static int noalloc_scratch(void** out) {
  static std::mutex mu;
  static void* ptrs[64] = {nullptr};
  int dev = 0;
  int st = check_cuda(cudaGetDevice(&dev), "attention (no-alloc): current device");
  if (st) return st;
  if (dev < 0 || dev >= 64)
    return set_error(TM_ERR_UNSUPPORTED, "attention (no-alloc): device %d out of range", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    st = check_cuda(cudaGetSymbolAddress(&p, g_noalloc_scratch),
                    "attention (no-alloc): address of the fixed scratch");
    if (st) return st;
    ptrs[dev] = p;
  }
  *out = ptrs[dev];
  return TM_OK;
}

}  // namespace attn
}  // namespace tmb

extern "C" int tm_attention_fwd_noalloc(const void* q, int64_t q_batch_stride,
                                        int64_t q_row_stride, const void* k_cache,
                                        const void* v_cache, int64_t cache_batch_stride,
                                        int64_t cache_row_stride, int64_t cache_rows,
                                        const void* k_new, const void* v_new,
                                        int64_t new_batch_stride, int64_t new_row_stride,
                                        int64_t new_rows, const tm_kv_span* spans, int n_spans,
                                        void* out, int64_t out_batch_stride,
                                        int64_t out_row_stride, int B, int Lq, int H, int D,
                                        float scale, void* stream) {
  using namespace tmb::attn;
  if (!spans || n_spans < 1)
    return set_error(TM_ERR_INVALID_ARGUMENT, "attention: null pointer or no spans");
  if (D != 64 && D != 128) return set_error(TM_ERR_UNSUPPORTED, "attention: head dim %d", D);
  if (B < 1 || Lq < 1 || H < 1)
    return set_error(TM_ERR_INVALID_ARGUMENT, "attention: B=%d Lq=%d H=%d", B, Lq, H);
  // The scratch need of the work partition the launch will choose: planned
  // from the same key-tile list (each span starts a new tile) with no cap.
  int2 tiles[kMaxTiles];
  bool use_src[2] = {false, false};
  int nt = 0;
  const int st_tiles = build_tiles(spans, n_spans, cache_rows, new_rows, tiles, &nt, use_src);
  if (st_tiles) return st_tiles;
  const int64_t need =
      split_ws_bytes(make_plan(B, Lq, H, D, nt, INT64_MAX).kv_splits, B, Lq, H, D);
  if (need > kNoAllocScratchBytes)
    return set_error(TM_ERR_INVALID_ARGUMENT,
                     "attention (no-alloc): B=%d Lq=%d H=%d D=%d over %d key tiles needs %lld "
                     "bytes of scratch, above the fixed %lld bytes; use tm_attention_fwd_ws",
                     B, Lq, H, D, nt, (long long)need,
                     (long long)kNoAllocScratchBytes);
  void* scratch = nullptr;
  const int st = noalloc_scratch(&scratch);
  if (st) return st;
  // Every row the merge pass reads is written first in the same call, so
  // nothing left in the array by an earlier call needs clearing.
  return attention_impl(q, q_batch_stride, q_row_stride, k_cache, v_cache, cache_batch_stride,
                        cache_row_stride, cache_rows, k_new, v_new, new_batch_stride,
                        new_row_stride, new_rows, spans, n_spans, out, out_batch_stride,
                        out_row_stride, B, Lq, H, D, scale,
                        ext_ws(scratch, kNoAllocScratchBytes), stream);
}
