// Block-causal streaming attention on sm_100a tensor cores.
//
// One CTA computes a 128-row query tile of one (batch, head) against the
// ordered list of visible key tiles (anchor + rolling window from the slot
// arena, then the current chunk).  The key tiles are split between two
// softmax warpgroups ("lanes"): lane 0 takes the first ceil(n/2) tiles, lane
// 1 the rest, and the two partial results are merged at the end, so the
// tensor core works on one lane's QK^T / PV while the other lane runs its
// softmax.  Warp roles (12 warps, 3 warpgroups):
//   warp 0      TMA producer: Q once, then K and V tiles (lane-interleaved
//               order) into separate rings; K runs one tile ahead of V.
//   warp 1      TMEM owner and tcgen05.mma issuer (one thread):
//               S_l = Q K^T into lane l's TMEM tile, O_l += P_l V with P_l read
//               from TMEM (TS form).
//   warps 2..3  idle (they hand their registers to the softmax warpgroups).
//   warps 4..7  lane 0 softmax, warps 8..11 lane 1 softmax: thread r of a
//               warpgroup owns query row r (its TMEM lane); it reads its S row,
//               keeps the running max / sum in registers, writes P (bf16) back
//               over S in TMEM, and rescales O_l in TMEM only when the running
//               max grows by more than 2^8 (the final division uses the same
//               reference max, so the result is exact).
//   lane 0 then merges lane 1's (O, max, sum) and writes O / sum as bf16.
//
// TMEM: S0/P0 [0,128), S1/P1 [128,256), O0 [256,256+D), O1 [256+D,256+2D).
// Visibility (anchor + window + chunk) arrives as a host-built list of key
// tiles, each (source, first row, valid rows); keys beyond `valid` are masked
// to -inf in registers, nothing is materialised.
//
// Reference semantics: softmax(Q K^T / sqrt(D)) V without a mask over
// cat(cached, new) (ltx_causal/transformer/kv_cache.py:1486-1531,
// ltx_causal/attention/flex_attention_utils.py:225-276).
#include <cmath>
#include <vector>

#include "common.cuh"
#include "host_common.h"

namespace tmb {
namespace attn {

constexpr int BM = 128;          // query rows per CTA (one TMEM lane each)
constexpr int BN = 128;          // keys per tile
constexpr int kMaxTiles = 192;   // 24576 visible keys
constexpr int kThreads = 384;    // 12 warps
// Register split (setmaxnreg): launched at 168 per thread (384 x 168 =
// 64512); warpgroup 0 drops to 88, the two softmax warpgroups rise to 208:
// 128 x 88 + 256 x 208 = 64512, the launch total.
constexpr int kRegsCtrl = 88;
constexpr int kRegsSoftmax = 208;

struct __align__(64) Params {
  CUtensorMap tm_q;
  CUtensorMap tm_k[2];  // [TM_KV_SOURCE_CACHE], [TM_KV_SOURCE_NEW]
  CUtensorMap tm_v[2];
  int2 tiles[kMaxTiles];  // x = (source << 30) | first row, y = valid rows (1..BN)
  int n_tiles;
  int Lq;
  int64_t out_bs, out_rs;  // elements
  __nv_bfloat16* out;
  float scale_log2;
  int* err;
};

template <int D>
struct Cfg {
  static constexpr int kKStages = 3;
  static constexpr int kVStages = (D == 128) ? 2 : 3;
  static constexpr int kBlk = 128 * 128;  // bytes of one 128-row x 64-col swizzle block
  static constexpr int kQBytes = BM * D * 2;
  static constexpr int kKVBytes = BN * D * 2;
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + kQBytes;
  static constexpr int kVOff = kKOff + kKStages * kKVBytes;
  static constexpr int kBarOff = kVOff + kVStages * kKVBytes;
  // barriers: q_full, k_full[KS], k_empty[KS], v_full[VS], v_empty[VS],
  //           s_full[2], p_full[2], pv_done[2], drain
  static constexpr int kNumBars = 1 + 2 * kKStages + 2 * kVStages + 6 + 1;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;  // tmem slot, abort flag
  static constexpr int kMLOff = kMiscOff + 16;             // lane-1 max / sum per row
  static constexpr int kSmemBytes = kMLOff + 2 * BM * 4;
  static constexpr int kSmemAlloc = kSmemBytes + 1024;     // runtime 1 KB alignment slack
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kOCol = 256;                   // O_l at kOCol + l * D
};

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
  const int q_tile = blockIdx.x, head = blockIdx.y, batch = blockIdx.z;
  const int n = p.n_tiles;
  const int n0 = (n + 1) >> 1;  // lane 0 tiles [0, n0), lane 1 tiles [n0, n)
  const int n1 = n - n0;

  const uint32_t bar0 = sbase + C::kBarOff;
  const uint32_t b_q = bar0;
  auto b_kfull = [&](int s) { return bar0 + 8u * (1 + s); };
  auto b_kempty = [&](int s) { return bar0 + 8u * (1 + KS + s); };
  auto b_vfull = [&](int s) { return bar0 + 8u * (1 + 2 * KS + s); };
  auto b_vempty = [&](int s) { return bar0 + 8u * (1 + 2 * KS + VS + s); };
  const uint32_t bar1 = bar0 + 8u * (1 + 2 * KS + 2 * VS);
  auto b_sfull = [&](int l) { return bar1 + 8u * l; };
  auto b_pfull = [&](int l) { return bar1 + 8u * (2 + l); };
  auto b_pvdone = [&](int l) { return bar1 + 8u * (4 + l); };
  const uint32_t b_drain = bar1 + 8u * 6;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kMiscOff + 4);
  float* m1_smem = reinterpret_cast<float*>(smem + C::kMLOff);
  float* l1_smem = m1_smem + BM;

  // item g (consumption order) -> tile: rounds of (lane 0, lane 1)
  auto tile_of = [&](int g) { return (g & 1) ? n0 + (g >> 1) : (g >> 1); };

  if (threadIdx.x == 0) {
    mbar_init(b_q, 1);
    for (int s = 0; s < KS; ++s) {
      mbar_init(b_kfull(s), 1);
      mbar_init(b_kempty(s), 1);
    }
    for (int s = 0; s < VS; ++s) {
      mbar_init(b_vfull(s), 1);
      mbar_init(b_vempty(s), 1);
    }
    for (int l = 0; l < 2; ++l) {
      mbar_init(b_sfull(l), 1);
      mbar_init(b_pfull(l), 128);
      mbar_init(b_pvdone(l), 1);
    }
    mbar_init(b_drain, 1);
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

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    if (lane_id == 0) {
      constexpr int kDB = D / 64;
      mbar_arrive_expect_tx(b_q, C::kQBytes);
      for (int db = 0; db < kDB; ++db)
        tma_load_4d(sbase + C::kQOff + db * C::kBlk, &p.tm_q, b_q, db * 64, head, q_tile * BM,
                    batch);
      auto load = [&](int g, bool is_k) -> bool {
        const int S = is_k ? KS : VS;
        const int s = g % S;
        if (g >= S && !mbar_wait(is_k ? b_kempty(s) : b_vempty(s), ((g / S) - 1) & 1, abort_flag,
                                 p.err))
          return false;
        const int2 tile = p.tiles[tile_of(g)];
        const int src = tile.x >> 30;
        const int row = tile.x & 0x3FFFFFFF;
        const uint32_t full = is_k ? b_kfull(s) : b_vfull(s);
        const uint32_t dst = sbase + (is_k ? C::kKOff : C::kVOff) + s * C::kKVBytes;
        const CUtensorMap* map = is_k ? &p.tm_k[src] : &p.tm_v[src];
        mbar_arrive_expect_tx(full, C::kKVBytes);
        for (int db = 0; db < kDB; ++db)
          tma_load_4d(dst + db * C::kBlk, map, full, db * 64, head, row, batch);
        return true;
      };
      int last_k = -1, last_v = -1;
      for (int g = 0; g <= n; ++g) {
        if (g < n) {
          if (!load(g, true)) break;
          last_k = g;
        }
        if (g >= 1) {
          if (!load(g - 1, false)) break;
          last_v = g - 1;
        }
      }
      if (*abort_flag) {
        // Let every issued copy land before the CTA's shared memory is released.
        mbar_wait(b_q, 0, nullptr, p.err, 100000000ull);
        for (int g = last_k - KS + 1; g <= last_k; ++g)
          if (g >= 0) mbar_wait(b_kfull(g % KS), (g / KS) & 1, nullptr, p.err, 100000000ull);
        for (int g = last_v - VS + 1; g <= last_v; ++g)
          if (g >= 0) mbar_wait(b_vfull(g % VS), (g / VS) & 1, nullptr, p.err, 100000000ull);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane_id == 0) {
      constexpr uint32_t idesc_qk = idesc_bf16_f32(BM, BN, 0);
      constexpr uint32_t idesc_pv = idesc_bf16_f32(BM, D, 1);
      bool ok = mbar_wait(b_q, 0, abort_flag, p.err);
      for (int j = 0; ok && j < n0; ++j) {
        for (int l = 0; l < 2 && ok; ++l) {
          const int g = 2 * j + l;
          if (g >= n) break;
          const int s = g % KS;
          if (!mbar_wait(b_kfull(s), (g / KS) & 1, abort_flag, p.err)) { ok = false; break; }
          // S_l / P_l is free once PV_l(j - 1) has completed.
          if (j >= 1 && !mbar_wait(b_pvdone(l), (j - 1) & 1, abort_flag, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t kbase = sbase + C::kKOff + s * C::kKVBytes;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint64_t a =
                smem_desc_sw128(sbase + C::kQOff + (kk >> 2) * C::kBlk + (kk & 3) * 32, 16, 1024);
            const uint64_t b =
                smem_desc_sw128(kbase + (kk >> 2) * C::kBlk + (kk & 3) * 32, 16, 1024);
            umma_ss(tmem + l * BN, a, b, idesc_qk, kk > 0 ? 1u : 0u);
          }
          umma_commit(b_sfull(l));
          umma_commit(b_kempty(s));
        }
        for (int l = 0; l < 2 && ok; ++l) {
          const int g = 2 * j + l;
          if (g >= n) break;
          const int sv = g % VS;
          if (!mbar_wait(b_pfull(l), j & 1, abort_flag, p.err)) { ok = false; break; }
          if (!mbar_wait(b_vfull(sv), (g / VS) & 1, abort_flag, p.err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t vbase = sbase + C::kVOff + sv * C::kKVBytes;
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            const uint64_t b = smem_desc_sw128(vbase + kk * 2048, C::kBlk, 1024);
            umma_ts(tmem + C::kOCol + l * D, tmem + l * BN + kk * 8, b, idesc_pv,
                    (j > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(b_pvdone(l));
          umma_commit(b_vempty(sv));
        }
      }
      if (!ok) {
        // Drain: wait for every issued MMA before TMEM is released.
        umma_commit(b_drain);
        mbar_wait(b_drain, 0, nullptr, p.err, 100000000ull);
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ softmax lanes
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));
    const int ln = (warp - 4) >> 2;  // 0 for warps 4..7, 1 for warps 8..11
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane_id;
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(q4 * 32) << 16);
    const uint32_t tS = t_lane + ln * BN;
    const uint32_t tO = t_lane + C::kOCol + ln * D;
    const int my_n = ln == 0 ? n0 : n1;
    const int tile0 = ln == 0 ? 0 : n0;
    const float sl = p.scale_log2;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    auto wait_all = [&](uint32_t bar, uint32_t par) -> bool {
      bool w = mbar_wait(bar, par, abort_flag, p.err);
      return __shfl_sync(0xffffffffu, w ? 1 : 0, 0) != 0;
    };
    for (int j = 0; j < my_n; ++j) {
      if (!wait_all(b_sfull(ln), j & 1)) { ok = false; break; }
      tc_fence_after();
      uint32_t sr[BN];
      TM_TMEM_LD32(tS + 0, (sr + 0));
      TM_TMEM_LD32(tS + 32, (sr + 32));
      TM_TMEM_LD32(tS + 64, (sr + 64));
      TM_TMEM_LD32(tS + 96, (sr + 96));
      tmem_wait_ld();

      const int valid = p.tiles[tile0 + j].y;
      if (valid < BN) {
#pragma unroll
        for (int c = 0; c < BN; ++c)
          if (c >= valid) sr[c] = __float_as_uint(-INFINITY);
      }
      float mx = fmax3f(__uint_as_float(sr[0]), __uint_as_float(sr[1]), __uint_as_float(sr[2]));
#pragma unroll
      for (int c = 3; c < BN - 1; c += 2)
        mx = fmax3f(mx, __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]));
      mx = fmaxf(mx, __uint_as_float(sr[BN - 1]));
      const float mx_s = mx * sl;
      bool need = false;
      float m_new = m_run;
      if (j == 0) {
        m_run = mx_s;
      } else if (mx_s > m_run + 8.0f) {
        need = true;
        m_new = mx_s;
      }
      if (__any_sync(0xffffffffu, need)) {
        // O_l must hold PV_l(j - 1) before it is rescaled.
        if (!wait_all(b_pvdone(ln), (j - 1) & 1)) { ok = false; break; }
        tc_fence_after();
        const float alpha = need ? ex2_approx(m_run - m_new) : 1.0f;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          TM_TMEM_LD32(tO + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          TM_TMEM_ST32(tO + c * 32, o);
        }
        tmem_wait_st();
        l_run *= alpha;
        m_run = m_new;
      }
      const uint64_t sl2 = f2_packf(sl, sl);
      const uint64_t nm2 = f2_packf(-m_run, -m_run);
      uint64_t acc[4] = {0, 0, 0, 0};
      uint32_t pk[BN / 2];
#pragma unroll
      for (int c = 0; c < BN; c += 2) {
        float x0, x1;
        f2_unpack(f2_fma(f2_pack(sr[c], sr[c + 1]), sl2, nm2), x0, x1);
        const float p0 = ex2_approx(x0);
        const float p1 = ex2_approx(x1);
        acc[(c >> 1) & 3] = f2_add(acc[(c >> 1) & 3], f2_packf(p0, p1));
        pk[c >> 1] = pack_bf16x2(p0, p1);
      }
      float a0, a1, a2, a3;
      f2_unpack(f2_add(acc[0], acc[1]), a0, a1);
      f2_unpack(f2_add(acc[2], acc[3]), a2, a3);
      l_run += (a0 + a1) + (a2 + a3);
      // P_l overwrites the first 64 columns of S_l (S is already in registers).
      TM_TMEM_ST32(tS + 0, (pk + 0));
      TM_TMEM_ST32(tS + 32, (pk + 32));
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(b_pfull(ln));
    }
    // the final PV of this lane
    const bool fin = ok && my_n > 0 && wait_all(b_pvdone(ln), (my_n - 1) & 1);
    if (ln == 1) {
      m1_smem[row] = fin ? m_run : -INFINITY;
      l1_smem[row] = fin ? l_run : 0.f;
    }
    named_bar_sync(1, 256);
    if (ln == 0 && fin) {
      // lane 1 has finished all its PV (it waited before the barrier), or had none
      const bool ok1 = (n1 == 0) || wait_all(b_pvdone(1), (n1 - 1) & 1);
      if (ok1) {
        tc_fence_after();
        const float m1 = m1_smem[row], l1 = l1_smem[row];
        const float m = fmaxf(m_run, m1);
        const float c0 = ex2_approx(m_run - m);
        const float c1 = (n1 > 0 && l1 > 0.f) ? ex2_approx(m1 - m) : 0.f;
        const float inv = 1.0f / (l_run * c0 + l1 * c1);
        const float s0 = c0 * inv, s1 = c1 * inv;
        const int qi = q_tile * BM + row;
        __nv_bfloat16* orow = p.out + static_cast<int64_t>(batch) * p.out_bs +
                              static_cast<int64_t>(qi) * p.out_rs +
                              static_cast<int64_t>(head) * D;
        const uint32_t tO1 = t_lane + C::kOCol + D;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32], o1[32];
          TM_TMEM_LD32(tO + c * 32, o);
          if (n1 > 0) {
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

// Encode a [B, rows, H, D] bf16 tensor (heads contiguous) as a 4-D TMA map
// with a {64, 1, 128, 1} box and 128-byte swizzle.
static int make_map(CUtensorMap* m, const void* base, int64_t rows, int B, int H, int D,
                    int64_t batch_stride, int64_t row_stride, const char* what) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return set_error(TM_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (B == 1) batch_stride = rows * row_stride;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(H),
                        static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(B)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(D) * 2, static_cast<cuuint64_t>(row_stride) * 2,
                           static_cast<cuuint64_t>(batch_stride) * 2};
  cuuint32_t box[4] = {64, 1, 128, 1};
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
  dim3 grid((Lq + BM - 1) / BM, H, B);
  attn_fwd_kernel<D><<<grid, kThreads, C::kSmemAlloc, stream>>>(prm);
  return check_cuda(cudaGetLastError(), "attention: launch");
}

}  // namespace attn
}  // namespace tmb

using namespace tmb;

extern "C" int tm_attention_fwd(const void* q, int64_t q_batch_stride, int64_t q_row_stride,
                                const void* k_cache, const void* v_cache,
                                int64_t cache_batch_stride, int64_t cache_row_stride,
                                int64_t cache_rows, const void* k_new, const void* v_new,
                                int64_t new_batch_stride, int64_t new_row_stride, int64_t new_rows,
                                const tm_kv_span* spans, int n_spans, void* out,
                                int64_t out_batch_stride, int64_t out_row_stride, int B, int Lq,
                                int H, int D, float scale, void* stream) {
  using namespace tmb::attn;
  if (D != 64 && D != 128) return set_error(TM_ERR_UNSUPPORTED, "attention: head dim %d", D);
  if (B < 1 || Lq < 1 || H < 1 || B > 65535 || H > 65535)
    return set_error(TM_ERR_INVALID_ARGUMENT, "attention: B=%d Lq=%d H=%d", B, Lq, H);
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
      prm.tiles[nt].x = (s.source << 30) | (s.row_start + off);
      prm.tiles[nt].y = (s.rows - off) < BN ? (s.rows - off) : BN;
      ++nt;
    }
    total += s.rows;
  }
  if (total == 0) return set_error(TM_ERR_INVALID_ARGUMENT, "attention: no visible keys");
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
  int st = make_map(&prm.tm_q, q, Lq, B, H, D, q_batch_stride, q_row_stride, "q");
  if (st) return st;
  for (int s = 0; s < 2; ++s) {
    const int src = use_src[s] ? s : (use_src[0] ? 0 : 1);  // unused slot: copy a valid map
    st = make_map(&prm.tm_k[s], kp[src], rows_of[src], B, H, D, bs_of[src], rs_of[src], "k");
    if (st) return st;
    st = make_map(&prm.tm_v[s], vp[src], rows_of[src], B, H, D, bs_of[src], rs_of[src], "v");
    if (st) return st;
  }
  prm.n_tiles = nt;
  prm.Lq = Lq;
  prm.out = static_cast<__nv_bfloat16*>(out);
  prm.out_bs = (B == 1) ? 0 : out_batch_stride;
  prm.out_rs = out_row_stride;
  const double sc = (scale > 0.f) ? (double)scale : 1.0 / std::sqrt((double)D);
  prm.scale_log2 = static_cast<float>(sc * 1.4426950408889634);
  prm.err = device_error_flag();
  if (!prm.err) return set_error(TM_ERR_CUDA, "attention: device error flag unavailable");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return D == 128 ? launch<128>(prm, B, Lq, H, s) : launch<64>(prm, B, Lq, H, s);
}
