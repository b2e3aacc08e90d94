// RoPE kernels: SPLIT cos/sin table generation (A1) and the fused q/k
// RMSNorm + split rotary + layout kernel (A2 + A3, optional Ulysses pack).
#include <cmath>

#include "common.cuh"
#include "host_common.h"

namespace tmb {
namespace rope {

// ---------------------------------------------------------------------------
// A1: tables.  The rotation angle is formed in fp32 with the reference's
// operation order (ltx_causal/rope/causal_rope.py:45-80, 253-308):
//   lin   = linspace(0, 1, n_freq)           (two-sided, one rounding each)
//   ind   = powf(theta, lin) * fp32(pi) / 2
//   frac  = physical position / max_pos      (fp32 divisions)
//   angle = ind * (2 frac - 1)
// laid out [f0_ax0, f0_ax1, f0_ax2, f1_ax0, ...] with `pad` identity entries in
// front, then split per head.
// ---------------------------------------------------------------------------
struct TableParams {
  void* cos_out;
  void* sin_out;
  int out_f32;
  int n_pos;
  int64_t g[3];
  int hp;      // entries per head (dim / 2 / heads)
  int heads;
  int pad;     // identity entries in front
  int n_freq;  // dim / (2 n_pos)
  float theta;
  float max_pos[3];
  int64_t start;
  int is_audio;
  int64_t repeat;
  int64_t T;   // tokens = prod(g) * repeat
};

__device__ __forceinline__ float temporal_seconds(float lt, int is_audio) {
  if (is_audio) {
    const float s = fmaxf(lt * 4.0f + 1.0f - 4.0f, 0.0f);
    const float e = fmaxf((lt + 1.0f) * 4.0f + 1.0f - 4.0f, 0.0f);
    return __fdiv_rn(__fmul_rn(__fdiv_rn(s + e, 2.0f), 160.0f), 16000.0f);
  }
  const float s = fmaxf(lt * 8.0f + 1.0f - 8.0f, 0.0f);
  const float e = fmaxf((lt + 1.0f) * 8.0f + 1.0f - 8.0f, 0.0f);
  return __fdiv_rn(__fdiv_rn(s + e, 2.0f), 24.0f);
}

__global__ void tables_kernel(const TableParams p) {
  const int64_t total = static_cast<int64_t>(p.heads) * p.T * p.hp;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int j = static_cast<int>(idx % p.hp);
    const int64_t t = (idx / p.hp) % p.T;
    const int h = static_cast<int>(idx / (static_cast<int64_t>(p.hp) * p.T));
    const int e = h * p.hp + j;
    float c = 1.0f, s = 0.0f;
    if (e >= p.pad) {
      const int k = e - p.pad;
      const int fi = k / p.n_pos;
      const int axis = k % p.n_pos;
      float lin;
      if (p.n_freq == 1) {
        lin = 0.0f;
      } else {
        const float step = __fdiv_rn(1.0f, static_cast<float>(p.n_freq - 1));
        lin = (fi < p.n_freq / 2) ? __fmaf_rn(step, static_cast<float>(fi), 0.0f)
                                  : __fmaf_rn(-step, static_cast<float>(p.n_freq - 1 - fi), 1.0f);
      }
      const float ind = __fdiv_rn(__fmul_rn(powf(p.theta, lin), 3.14159265358979323846f), 2.0f);
      const int64_t tb = t / p.repeat;
      float frac;
      if (p.n_pos == 3) {
        const int64_t hw = p.g[1] * p.g[2];
        if (axis == 0) {
          frac = __fdiv_rn(temporal_seconds(static_cast<float>(p.start + tb / hw), 0),
                           p.max_pos[0]);
        } else {
          const int64_t i = (axis == 1) ? (tb / p.g[2]) % p.g[1] : tb % p.g[2];
          frac = __fdiv_rn(static_cast<float>(i) * 32.0f + 16.0f, p.max_pos[axis]);
        }
      } else {
        frac = __fdiv_rn(temporal_seconds(static_cast<float>(p.start + tb), p.is_audio),
                         p.max_pos[0]);
      }
      const float angle = __fmul_rn(ind, __fsub_rn(__fmul_rn(frac, 2.0f), 1.0f));
      sincosf(angle, &s, &c);
    }
    if (p.out_f32) {
      static_cast<float*>(p.cos_out)[idx] = c;
      static_cast<float*>(p.sin_out)[idx] = s;
    } else {
      static_cast<__nv_bfloat16*>(p.cos_out)[idx] = __float2bfloat16_rn(c);
      static_cast<__nv_bfloat16*>(p.sin_out)[idx] = __float2bfloat16_rn(s);
    }
  }
}

// ---------------------------------------------------------------------------
// A2 + A3: one block of TPR = H*D / (8 * CPT) threads per token row; thread t
// handles the 16-byte chunks c = k * TPR + t (k < CPT), so every load
// instruction of a warp covers 512 contiguous bytes and all of a thread's loads
// (x, weight, cos, sin) are independent and issued up front.  Within a head of
// D/8 chunks, rotate-half pairs chunk j with chunk j +- D/16, held by thread
// t ^ (D/16) of the same warp.  The sum of squares is reduced over the block.
// ---------------------------------------------------------------------------
constexpr int kMaxJobs = 4;

struct Job {
  const __nv_bfloat16* x;
  __nv_bfloat16* out;
  const __nv_bfloat16* w;
  const __nv_bfloat16* cos;
  const __nv_bfloat16* sin;
  int64_t xbs, xrs, ogs, obs, ors, pbs, phs, prs;
  int64_t L;
};

struct NormRopeParams {
  Job jobs[kMaxJobs];
  int64_t row_begin[kMaxJobs + 1];  // prefix sums of B * L
  int64_t delta[8];  // bytes from a job's output address to head group g's owner (peer store)
  int n_jobs;
  int B, H;
  float eps;
  int sp;
};

__device__ __forceinline__ void unpack8(const uint4& v, float* f) {
  const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(u[i] << 16);
    f[2 * i + 1] = __uint_as_float(u[i] & 0xFFFF0000u);
  }
}

// At least 6 blocks per SM (79 registers at H*D = 4096 instead of 96, no
// spills): one more row in flight per SM; measured 19.8 vs 21.8 us per call
// in the C2 step.
template <int D, int CPT, int TPR>
__global__ void __launch_bounds__(TPR, 6)
    norm_rope_kernel(const __grid_constant__ NormRopeParams p) {
  constexpr int kChunksPerHead = D / 8;
  constexpr int kHalf = D / 16;
  constexpr int kInner = CPT * TPR * 8;
  constexpr int kWarps = TPR / 32;
  __shared__ float red[kWarps];
  const int t = threadIdx.x;
  const int lane = t & 31;
  const int64_t row = blockIdx.x;
  int ji = 0;
#pragma unroll
  for (int i = 1; i < kMaxJobs; ++i)
    if (i < p.n_jobs && row >= p.row_begin[i]) ji = i;
  const Job& jb = p.jobs[ji];
  const int64_t r = row - p.row_begin[ji];
  const int64_t b = r / jb.L;
  const int64_t l = r % jb.L;
  const int j = t % kChunksPerHead;  // chunk position within its head (same for every k)
  const bool first_half = j < kHalf;

  const __nv_bfloat16* xrow = jb.x + b * jb.xbs + l * jb.xrs;
  uint4 xr[CPT], cr[CPT], sr[CPT], wr[CPT];
#pragma unroll
  for (int k = 0; k < CPT; ++k) {
    const int c = k * TPR + t;
    xr[k] = *reinterpret_cast<const uint4*>(xrow + c * 8);
    if (jb.w != nullptr) wr[k] = __ldg(reinterpret_cast<const uint4*>(jb.w + c * 8));
    if (jb.cos != nullptr) {
      const int h = c / kChunksPerHead;
      const int64_t pe_off = b * jb.pbs + h * jb.phs + l * jb.prs + (j % kHalf) * 8;
      cr[k] = *reinterpret_cast<const uint4*>(jb.cos + pe_off);
      sr[k] = *reinterpret_cast<const uint4*>(jb.sin + pe_off);
    }
  }
  float rs = 1.0f;
  if (jb.w != nullptr) {
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < CPT; ++k) {
      float f[8];
      unpack8(xr[k], f);
#pragma unroll
      for (int i = 0; i < 8; ++i) ss = fmaf(f[i], f[i], ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (kWarps > 1) {
      if (lane == 0) red[t >> 5] = ss;
      __syncthreads();
      ss = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) ss += red[w];
    }
    rs = rsqrtf(ss / static_cast<float>(kInner) + p.eps);
  }
  const int Hl = p.H / p.sp;
#pragma unroll
  for (int k = 0; k < CPT; ++k) {
    const int c = k * TPR + t;
    const int h = c / kChunksPerHead;
    float y[8];
    unpack8(xr[k], y);
    if (jb.w != nullptr) {
      float w[8];
      unpack8(wr[k], w);
#pragma unroll
      for (int i = 0; i < 8; ++i) y[i] = y[i] * rs * w[i];
    }
    float o[8];
    if (jb.cos != nullptr) {
      float cs[8], sn[8], part[8];
      unpack8(cr[k], cs);
      unpack8(sr[k], sn);
#pragma unroll
      for (int i = 0; i < 8; ++i) part[i] = __shfl_xor_sync(0xffffffffu, y[i], kHalf);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        o[i] = first_half ? fmaf(y[i], cs[i], -part[i] * sn[i]) : fmaf(y[i], cs[i], part[i] * sn[i]);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = y[i];
    }
    const uint4 v = make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]),
                               pack_bf16x2(o[4], o[5]), pack_bf16x2(o[6], o[7]));
    const int g = h / Hl;
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(
        reinterpret_cast<char*>(jb.out + g * jb.ogs + b * jb.obs + l * jb.ors +
                                static_cast<int64_t>(h - g * Hl) * D + j * 8) +
        p.delta[g]);
    *reinterpret_cast<uint4*>(dst) = v;
  }
}

template <int D, int CPT, int TPR>
static int launch_norm_rope(const NormRopeParams& prm, cudaStream_t s) {
  const int64_t rows = prm.row_begin[prm.n_jobs];
  norm_rope_kernel<D, CPT, TPR><<<static_cast<unsigned>(rows), TPR, 0, s>>>(prm);
  return check_cuda(cudaGetLastError(), "norm_rope: launch");
}

}  // namespace rope
}  // namespace tmb

using namespace tmb;

extern "C" int tm_rope_tables_split(void* cos_out, void* sin_out, int out_dtype, int n_pos,
                                    const int64_t* grid, int dim, int num_heads, double theta,
                                    const double* max_pos, int64_t start_frame, int is_audio,
                                    int64_t repeat_per_frame, void* stream) {
  if (!cos_out || !sin_out || !grid || !max_pos)
    return set_error(TM_ERR_INVALID_ARGUMENT, "rope_tables: null pointer");
  if (n_pos != 1 && n_pos != 3)
    return set_error(TM_ERR_INVALID_ARGUMENT, "rope_tables: Unsupported num_pos_dims: %d", n_pos);
  if (out_dtype != TM_DTYPE_BF16 && out_dtype != TM_DTYPE_F32)
    return set_error(TM_ERR_UNSUPPORTED, "rope_tables: dtype %d", out_dtype);
  if (dim <= 0 || num_heads <= 0 || (dim / 2) % num_heads != 0 || dim / (2 * n_pos) < 1)
    return set_error(TM_ERR_INVALID_ARGUMENT, "rope_tables: dim %d heads %d", dim, num_heads);
  if (repeat_per_frame < 1 || start_frame < 0 || start_frame > (1 << 22))
    return set_error(TM_ERR_INVALID_ARGUMENT, "rope_tables: repeat %lld start %lld",
                     (long long)repeat_per_frame, (long long)start_frame);
  rope::TableParams p;
  memset(&p, 0, sizeof(p));
  p.cos_out = cos_out;
  p.sin_out = sin_out;
  p.out_f32 = out_dtype == TM_DTYPE_F32;
  p.n_pos = n_pos;
  int64_t prod = 1;
  for (int i = 0; i < n_pos; ++i) {
    if (grid[i] < 1) return set_error(TM_ERR_INVALID_ARGUMENT, "rope_tables: grid[%d] < 1", i);
    p.g[i] = grid[i];
    p.max_pos[i] = static_cast<float>(max_pos[i]);
    prod *= grid[i];
  }
  p.n_freq = dim / (2 * n_pos);
  p.pad = dim / 2 - p.n_freq * n_pos;
  p.hp = dim / 2 / num_heads;
  p.heads = num_heads;
  p.theta = static_cast<float>(theta);
  p.start = start_frame;
  p.is_audio = is_audio ? 1 : 0;
  p.repeat = repeat_per_frame;
  p.T = prod * repeat_per_frame;
  const int64_t total = static_cast<int64_t>(num_heads) * p.T * p.hp;
  const int threads = 256;
  int64_t blocks = (total + threads - 1) / threads;
  if (blocks > 148 * 64) blocks = 148 * 64;
  rope::tables_kernel<<<static_cast<unsigned>(blocks), threads, 0,
                        static_cast<cudaStream_t>(stream)>>>(p);
  return check_cuda(cudaGetLastError(), "rope_tables: launch");
}

static int norm_rope_impl(const tm_norm_rope_job* jobs, int n_jobs, int B, int H, int D,
                          float eps, int sp_size, const int64_t* group_delta, void* stream) {
  using namespace tmb::rope;
  if (!jobs || n_jobs < 1 || n_jobs > kMaxJobs)
    return set_error(TM_ERR_INVALID_ARGUMENT, "norm_rope: %d jobs (1..%d)", n_jobs, kMaxJobs);
  if (D != 64 && D != 128) return set_error(TM_ERR_UNSUPPORTED, "norm_rope: head dim %d", D);
  const int inner = H * D;
  if (B < 1 || H < 1 || (inner != 256 && inner != 512 && inner != 1024 && inner != 2048 &&
                         inner != 4096))
    return set_error(TM_ERR_INVALID_ARGUMENT,
                     "norm_rope: H*D=%d must be 256, 512, 1024, 2048 or 4096", inner);
  if (sp_size < 1 || H % sp_size != 0)
    return set_error(TM_ERR_INVALID_ARGUMENT, "norm_rope: H (%d) must be divisible by sp_size (%d)",
                     H, sp_size);
  NormRopeParams p;
  memset(&p, 0, sizeof(p));
  p.n_jobs = n_jobs;
  p.B = B;
  p.H = H;
  p.eps = eps;
  p.sp = sp_size;
  int64_t acc = 0;
  for (int i = 0; i < n_jobs; ++i) {
    const tm_norm_rope_job& j = jobs[i];
    if (!j.x || !j.out || j.L < 1)
      return set_error(TM_ERR_INVALID_ARGUMENT, "norm_rope: job %d null or empty", i);
    if ((j.cos == nullptr) != (j.sin == nullptr))
      return set_error(TM_ERR_INVALID_ARGUMENT, "norm_rope: job %d has only one of cos/sin", i);
    const void* ptrs[5] = {j.x, j.out, j.norm_weight, j.cos, j.sin};
    for (int k = 0; k < 5; ++k)
      if (ptrs[k] && !aligned16(ptrs[k]))
        return set_error(TM_ERR_ALIGNMENT, "norm_rope: job %d pointer %d not 16-byte aligned", i,
                         k);
    const int64_t st[5] = {j.x_row_stride, j.x_batch_stride, j.out_row_stride,
                           j.out_batch_stride, j.out_group_stride};
    for (int k = 0; k < 5; ++k)
      if (st[k] & 7)
        return set_error(TM_ERR_ALIGNMENT, "norm_rope: job %d stride not a multiple of 8", i);
    if (j.cos && ((j.pe_row_stride & 7) || (j.pe_head_stride & 7) || (j.pe_batch_stride & 7)))
      return set_error(TM_ERR_ALIGNMENT, "norm_rope: job %d cos/sin stride not a multiple of 8",
                       i);
    Job& d = p.jobs[i];
    d.x = static_cast<const __nv_bfloat16*>(j.x);
    d.out = static_cast<__nv_bfloat16*>(j.out);
    d.w = static_cast<const __nv_bfloat16*>(j.norm_weight);
    d.cos = static_cast<const __nv_bfloat16*>(j.cos);
    d.sin = static_cast<const __nv_bfloat16*>(j.sin);
    d.xbs = j.x_batch_stride;
    d.xrs = j.x_row_stride;
    d.ogs = j.out_group_stride;
    d.obs = j.out_batch_stride;
    d.ors = j.out_row_stride;
    d.pbs = j.pe_batch_stride;
    d.phs = j.pe_head_stride;
    d.prs = j.pe_row_stride;
    d.L = j.L;
    p.row_begin[i] = acc;
    acc += static_cast<int64_t>(B) * j.L;
  }
  p.row_begin[n_jobs] = acc;
  if (group_delta) {
    if (sp_size > 8) return set_error(TM_ERR_UNSUPPORTED, "norm_rope: more than 8 peer groups");
    for (int g = 0; g < sp_size; ++g) {
      if (group_delta[g] & 15)
        return set_error(TM_ERR_ALIGNMENT, "norm_rope: peer offset %d not 16-byte aligned", g);
      p.delta[g] = group_delta[g];
    }
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (inner) {  // chunks per thread x threads per row = inner / 8
    case 256: return D == 128 ? launch_norm_rope<128, 1, 32>(p, s) : launch_norm_rope<64, 1, 32>(p, s);
    case 512: return D == 128 ? launch_norm_rope<128, 2, 32>(p, s) : launch_norm_rope<64, 2, 32>(p, s);
    case 1024: return D == 128 ? launch_norm_rope<128, 4, 32>(p, s) : launch_norm_rope<64, 4, 32>(p, s);
    case 2048: return D == 128 ? launch_norm_rope<128, 4, 64>(p, s) : launch_norm_rope<64, 4, 64>(p, s);
    case 4096: return D == 128 ? launch_norm_rope<128, 4, 128>(p, s) : launch_norm_rope<64, 4, 128>(p, s);
    default: break;
  }
  return set_error(TM_ERR_UNSUPPORTED, "norm_rope: H*D=%d not built", inner);
}

extern "C" int tm_norm_rope(const tm_norm_rope_job* jobs, int n_jobs, int B, int H, int D,
                            float eps, int sp_size, void* stream) {
  return norm_rope_impl(jobs, n_jobs, B, H, D, eps, sp_size, nullptr, stream);
}

extern "C" int tm_norm_rope_peer(const tm_norm_rope_job* jobs, int n_jobs, int B, int H, int D,
                                 float eps, int sp_size, const int64_t* group_delta,
                                 void* stream) {
  if (!group_delta) return set_error(TM_ERR_INVALID_ARGUMENT, "norm_rope_peer: null offsets");
  return norm_rope_impl(jobs, n_jobs, B, H, D, eps, sp_size, group_delta, stream);
}
