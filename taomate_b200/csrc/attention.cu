// Block-causal streaming attention on sm_100a tensor cores.
//
// One CTA computes a 128-row query tile of one (batch, head) against the
// ordered list of visible key tiles (anchor + rolling window from the slot
// arena, then the current chunk).  Warp roles:
//   warp 0      TMA producer: Q once, then K/V tiles into a STAGES-deep ring.
//   warp 1      TMEM owner and tcgen05.mma issuer (one elected thread):
//               S = Q K^T into a double-buffered TMEM tile, O += P V into a
//               TMEM accumulator.
//   warps 2..5  softmax: thread r of the warpgroup owns query row r (its TMEM
//               lane), reads its S row, keeps the running max / sum in
//               registers, writes P (bf16) into shared memory as the A
//               operand of the PV product, and rescales O in TMEM only when
//               the running max grows by more than 2^8 (lazy rescaling keeps
//               the result exact because the final division uses the same
//               reference max).  It also runs the epilogue O / l -> bf16.
//
// Visibility (anchor + window + chunk) arrives as a host-built list of key
// tiles, each (source, first row, valid rows).  Keys beyond `valid` in a tile
// are masked to -inf in registers, so nothing is materialised.
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
constexpr int kThreads = 192;    // 6 warps

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
  static constexpr int kStages = (D == 128) ? 2 : 3;
  static constexpr int kBlk = 128 * 128;            // bytes of one 128-row x 64-col swizzle block
  static constexpr int kQBytes = BM * D * 2;
  static constexpr int kKVBytes = BN * D * 2;
  static constexpr int kPBytes = BM * BN * 2;
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + kQBytes;
  static constexpr int kVOff = kKOff + kStages * kKVBytes;
  static constexpr int kPOff = kVOff + kStages * kKVBytes;
  static constexpr int kBarOff = kPOff + 2 * kPBytes;
  // barriers: q_full, k_full[S], v_full[S], k_empty[S], v_empty[S], s_full[2],
  //           s_empty[2], p_full[2], pv_done[2], drain
  static constexpr int kNumBars = 1 + 4 * kStages + 8 + 1;
  static constexpr int kSmemBytes = kBarOff + kNumBars * 8 + 16;
  static constexpr int kSmemAlloc = kSmemBytes + 1024;  // runtime 1 KB alignment slack
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kOCol = 256;              // S0 at 0, S1 at 128, O at 256
};

template <int D>
__global__ void __launch_bounds__(kThreads, 1) attn_fwd_kernel(const __grid_constant__ Params p) {
  using C = Cfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_addr(smem);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int q_tile = blockIdx.x, head = blockIdx.y, batch = blockIdx.z;
  const int n = p.n_tiles;

  const uint32_t bar0 = sbase + C::kBarOff;
  const uint32_t b_q = bar0;
  auto b_kfull = [&](int s) { return bar0 + 8u * (1 + s); };
  auto b_vfull = [&](int s) { return bar0 + 8u * (1 + C::kStages + s); };
  auto b_kempty = [&](int s) { return bar0 + 8u * (1 + 2 * C::kStages + s); };
  auto b_vempty = [&](int s) { return bar0 + 8u * (1 + 3 * C::kStages + s); };
  const uint32_t bar1 = bar0 + 8u * (1 + 4 * C::kStages);
  auto b_sfull = [&](int b) { return bar1 + 8u * b; };
  auto b_sempty = [&](int b) { return bar1 + 8u * (2 + b); };
  auto b_pfull = [&](int b) { return bar1 + 8u * (4 + b); };
  auto b_pvdone = [&](int b) { return bar1 + 8u * (6 + b); };
  const uint32_t b_drain = bar1 + 8u * 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kBarOff + C::kNumBars * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  if (threadIdx.x == 0) {
    mbar_init(b_q, 1);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(b_kfull(s), 1);
      mbar_init(b_vfull(s), 1);
      mbar_init(b_kempty(s), 1);
      mbar_init(b_vempty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(b_sfull(b), 1);
      mbar_init(b_sempty(b), 128);
      mbar_init(b_pfull(b), 128);
      mbar_init(b_pvdone(b), 1);
    }
    mbar_init(b_drain, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_addr(tmem_slot), C::kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
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

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      constexpr int kDB = D / 64;
      mbar_arrive_expect_tx(b_q, C::kQBytes);
      for (int db = 0; db < kDB; ++db)
        tma_load_4d(sbase + C::kQOff + db * C::kBlk, &p.tm_q, b_q, db * 64, head, q_tile * BM,
                    batch);
      // K runs one tile ahead of V: K(t) needs only QK(t - S) to be done,
      // V(t) needs PV(t - S).
      auto load_k = [&](int t) -> bool {
        const int s = t % C::kStages;
        if (t >= C::kStages &&
            !mbar_wait(b_kempty(s), ((t / C::kStages) - 1) & 1, abort_flag, p.err))
          return false;
        const int2 tile = p.tiles[t];
        const int src = tile.x >> 30;
        const int row = tile.x & 0x3FFFFFFF;
        mbar_arrive_expect_tx(b_kfull(s), C::kKVBytes);
        for (int db = 0; db < kDB; ++db)
          tma_load_4d(sbase + C::kKOff + s * C::kKVBytes + db * C::kBlk, &p.tm_k[src], b_kfull(s),
                      db * 64, head, row, batch);
        return true;
      };
      auto load_v = [&](int t) -> bool {
        const int s = t % C::kStages;
        if (t >= C::kStages &&
            !mbar_wait(b_vempty(s), ((t / C::kStages) - 1) & 1, abort_flag, p.err))
          return false;
        const int2 tile = p.tiles[t];
        const int src = tile.x >> 30;
        const int row = tile.x & 0x3FFFFFFF;
        mbar_arrive_expect_tx(b_vfull(s), C::kKVBytes);
        for (int db = 0; db < kDB; ++db)
          tma_load_4d(sbase + C::kVOff + s * C::kKVBytes + db * C::kBlk, &p.tm_v[src], b_vfull(s),
                      db * 64, head, row, batch);
        return true;
      };
      int last_k = -1, last_v = -1;
      for (int t = 0; t <= n; ++t) {
        if (t < n) {
          if (!load_k(t)) break;
          last_k = t;
        }
        if (t >= 1) {
          if (!load_v(t - 1)) break;
          last_v = t - 1;
        }
      }
      if (*abort_flag) {
        // Let every issued copy land before the CTA's shared memory is released.
        mbar_wait(b_q, 0, nullptr, p.err, 100000000ull);
        for (int t = last_k - C::kStages + 1; t <= last_k; ++t)
          if (t >= 0)
            mbar_wait(b_kfull(t % C::kStages), (t / C::kStages) & 1, nullptr, p.err, 100000000ull);
        for (int t = last_v - C::kStages + 1; t <= last_v; ++t)
          if (t >= 0)
            mbar_wait(b_vfull(t % C::kStages), (t / C::kStages) & 1, nullptr, p.err, 100000000ull);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = idesc_bf16_f32(BM, BN, 0);
      constexpr uint32_t idesc_pv = idesc_bf16_f32(BM, D, 1);
      auto issue_pv = [&](int j) -> bool {
        const int pb = j & 1;
        const int s = j % C::kStages;
        if (!mbar_wait(b_pfull(pb), (j >> 1) & 1, abort_flag, p.err)) return false;
        if (!mbar_wait(b_vfull(s), (j / C::kStages) & 1, abort_flag, p.err)) return false;
        tc_fence_after();
        const uint32_t pbase = sbase + C::kPOff + pb * C::kPBytes;
        const uint32_t vbase = sbase + C::kVOff + s * C::kKVBytes;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t a = smem_desc_sw128(pbase + (kk >> 2) * C::kBlk + (kk & 3) * 32, 16, 1024);
          const uint64_t b = smem_desc_sw128(vbase + kk * 2048, C::kBlk, 1024);
          umma_ss(tmem + C::kOCol, a, b, idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(b_pvdone(pb));
        umma_commit(b_vempty(s));
        return true;
      };
      bool ok = mbar_wait(b_q, 0, abort_flag, p.err);
      for (int t = 0; ok && t < n; ++t) {
        const int s = t % C::kStages;
        const int sb = t & 1;
        if (!mbar_wait(b_kfull(s), (t / C::kStages) & 1, abort_flag, p.err)) { ok = false; break; }
        if (t >= 2 && !mbar_wait(b_sempty(sb), ((t >> 1) - 1) & 1, abort_flag, p.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t kbase = sbase + C::kKOff + s * C::kKVBytes;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t a =
              smem_desc_sw128(sbase + C::kQOff + (kk >> 2) * C::kBlk + (kk & 3) * 32, 16, 1024);
          const uint64_t b = smem_desc_sw128(kbase + (kk >> 2) * C::kBlk + (kk & 3) * 32, 16, 1024);
          umma_ss(tmem + sb * BN, a, b, idesc_qk, kk > 0 ? 1u : 0u);
        }
        umma_commit(b_sfull(sb));
        umma_commit(b_kempty(s));
        if (t >= 1 && !issue_pv(t - 1)) { ok = false; break; }
      }
      if (ok && n > 0) ok = issue_pv(n - 1);
      if (!ok) {
        // Drain: wait for every issued MMA before TMEM is released.
        umma_commit(b_drain);
        mbar_wait(b_drain, 0, nullptr, p.err, 100000000ull);
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane;
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(q4 * 32) << 16);
    const float sl = p.scale_log2;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    auto wait_all = [&](uint32_t bar, uint32_t par) -> bool {
      bool w = mbar_wait(bar, par, abort_flag, p.err);
      return __shfl_sync(0xffffffffu, w ? 1 : 0, 0) != 0;
    };
    for (int t = 0; t < n; ++t) {
      const int sb = t & 1;
      if (!wait_all(b_sfull(sb), (t >> 1) & 1)) { ok = false; break; }
      tc_fence_after();
      uint32_t sr[BN];
      TM_TMEM_LD32(t_lane + sb * BN + 0, (sr + 0));
      TM_TMEM_LD32(t_lane + sb * BN + 32, (sr + 32));
      TM_TMEM_LD32(t_lane + sb * BN + 64, (sr + 64));
      TM_TMEM_LD32(t_lane + sb * BN + 96, (sr + 96));
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(b_sempty(sb));

      const int valid = p.tiles[t].y;
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < BN; ++j) {
        float v = __uint_as_float(sr[j]);
        if (j >= valid) v = -INFINITY;
        sr[j] = __float_as_uint(v);
        mx = fmaxf(mx, v);
      }
      const float mx_s = mx * sl;
      bool need = false;
      float m_new = m_run;
      if (t == 0) {
        m_new = mx_s;
        m_run = mx_s;
      } else if (mx_s > m_run + 8.0f) {
        need = true;
        m_new = mx_s;
      }
      if (__any_sync(0xffffffffu, need)) {
        // O must hold PV(t-1) before it is rescaled.
        if (!wait_all(b_pvdone((t - 1) & 1), ((t - 1) >> 1) & 1)) { ok = false; break; }
        tc_fence_after();
        const float alpha = need ? ex2_approx(m_run - m_new) : 1.0f;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          TM_TMEM_LD32(t_lane + C::kOCol + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) o[j] = __float_as_uint(__uint_as_float(o[j]) * alpha);
          TM_TMEM_ST32(t_lane + C::kOCol + c * 32, o);
        }
        tmem_wait_st();
        l_run *= alpha;
        m_run = m_new;
      }
      float sum = 0.f;
      uint32_t pk[BN / 2];
#pragma unroll
      for (int j = 0; j < BN; j += 2) {
        const float p0 = ex2_approx(fmaf(__uint_as_float(sr[j]), sl, -m_run));
        const float p1 = ex2_approx(fmaf(__uint_as_float(sr[j + 1]), sl, -m_run));
        sum += p0 + p1;
        pk[j >> 1] = pack_bf16x2(p0, p1);
      }
      l_run += sum;
      // P buffer sb is free once PV(t-2) has completed.
      if (t >= 2 && !wait_all(b_pvdone(sb), ((t >> 1) - 1) & 1)) { ok = false; break; }
      uint8_t* prow = smem + C::kPOff + sb * C::kPBytes + row * 128;
#pragma unroll
      for (int kb = 0; kb < 2; ++kb) {
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 v = make_uint4(pk[kb * 32 + c * 4 + 0], pk[kb * 32 + c * 4 + 1],
                                     pk[kb * 32 + c * 4 + 2], pk[kb * 32 + c * 4 + 3]);
          *reinterpret_cast<uint4*>(prow + kb * C::kBlk + ((c ^ (row & 7)) << 4)) = v;
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(b_pfull(sb));
    }
    if (ok && n > 0 && wait_all(b_pvdone((n - 1) & 1), ((n - 1) >> 1) & 1)) {
      tc_fence_after();
      const float inv_l = 1.0f / l_run;
      const int qi = q_tile * BM + row;
      __nv_bfloat16* orow = p.out + static_cast<int64_t>(batch) * p.out_bs +
                            static_cast<int64_t>(qi) * p.out_rs + static_cast<int64_t>(head) * D;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        TM_TMEM_LD32(t_lane + C::kOCol + c * 32, o);
        tmem_wait_ld();
        if (qi < p.Lq) {
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            const uint4 v = make_uint4(
                pack_bf16x2(__uint_as_float(o[j + 0]) * inv_l, __uint_as_float(o[j + 1]) * inv_l),
                pack_bf16x2(__uint_as_float(o[j + 2]) * inv_l, __uint_as_float(o[j + 3]) * inv_l),
                pack_bf16x2(__uint_as_float(o[j + 4]) * inv_l, __uint_as_float(o[j + 5]) * inv_l),
                pack_bf16x2(__uint_as_float(o[j + 6]) * inv_l, __uint_as_float(o[j + 7]) * inv_l));
            *reinterpret_cast<uint4*>(orow + c * 32 + j) = v;
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
