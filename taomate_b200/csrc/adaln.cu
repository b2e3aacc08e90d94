// Elementwise kernels of the transformer block around the attention: the
// gated residual update, RMSNorm / LayerNorm and the AdaLN modulation fused in
// one pass over a token row, and the tanh-approximate GELU of the FFN.
//
// Reference counterparts (ltx_causal/transformer/kv_cache.py,
// block_forward_with_cache, 2145-2654):
//   norm_vx = rms_norm(vx) * (1 + scale) + shift      (2200-2201, 2514-2525, 2604-2606)
//   vx = vx + out * gate                              (2217, 2566, 2610)
//   (scale, shift, gate) = table[i] + timestep[..., i, :]
//                                  (CausalAVTransformerBlock.get_ada_values,
//                                   ltx_causal/transformer/causal_block.py:434-452)
//   LayerNorm + (1 + scale) + shift before proj_out   (causal_model.py:568-598)
//   gelu(x, approximate="tanh")                        (transformer/compat.py:40)
//
// B200 layout: one CTA per token row, 16-byte loads and stores, every operand
// read once from HBM.  The AdaLN parameters are read per frame (row index
// (token + offset) / div), so the per-token expansion the reference
// materialises (kv_cache.py:2970: [B, L, 6 * D] per forward) is never built;
// the parameter rows are L2-resident.  All arithmetic in fp32, one bf16
// rounding per stored value.
#include <cuda_bf16.h>

#include "common.cuh"
#include "host_common.h"

namespace tmb {
namespace adaln {

struct Src {
  const __nv_bfloat16* table;  // [n, D] or null
  const __nv_bfloat16* ts;     // parameter rows, row stride ts_rs, or null
  int64_t ts_bs, ts_rs;
  int32_t ts_div, ts_off;
};

struct Params {
  const __nv_bfloat16* x;
  int64_t x_bs, x_rs;
  const __nv_bfloat16* y;
  int64_t y_bs, y_rs;
  __nv_bfloat16* xo;
  int64_t xo_bs, xo_rs;
  Src gate;
  int gate_idx;
  __nv_bfloat16* out[2];
  int64_t out_bs[2], out_rs[2];
  Src mod[2];
  int scale_idx[2], shift_idx[2];
  int n_out, norm_kind, L, D;
  float eps;
};

__device__ __forceinline__ void bf8_to_f32(const uint4& u, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 f32_to_bf8(const float* f) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return u;
}

// The parameter rows of one token row (b, t): the table and this token's
// timestep row (row (t + offset) / div, computed once per CTA).
struct Row {
  const __nv_bfloat16* table;
  const __nv_bfloat16* ts;
};

__device__ __forceinline__ Row param_row(const Src& s, int b, int t) {
  Row r{s.table, nullptr};
  if (s.ts) {
    const int row = (t + s.ts_off) / s.ts_div;  // 32-bit: token and frame indices fit
    r.ts = s.ts + b * s.ts_bs + static_cast<int64_t>(row) * s.ts_rs;
  }
  return r;
}

// value of parameter p at columns c..c+7: table[p] + ts_row[p]
__device__ __forceinline__ void param8(const Row& s, int p, int D, int c, float* out) {
#pragma unroll
  for (int i = 0; i < 8; ++i) out[i] = 0.f;
  float tmp[8];
  const int64_t off = static_cast<int64_t>(p) * D + c;
  if (s.table) {
    bf8_to_f32(__ldg(reinterpret_cast<const uint4*>(s.table + off)), tmp);
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i] += tmp[i];
  }
  if (s.ts) {
    bf8_to_f32(__ldg(reinterpret_cast<const uint4*>(s.ts + off)), tmp);
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i] += tmp[i];
  }
}

template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  constexpr int W = NT / 32;
  if (W == 1) return v;
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();  // red[] free (a previous reduction has been read)
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < W; ++i) s += red[i];
  return s;
}

// NT threads per row, CH 8-column chunks per thread: D = NT * CH * 8.
template <int NT, int CH>
__global__ void __launch_bounds__(NT, 4) residual_norm_kernel(const __grid_constant__ Params p) {
  __shared__ float red[NT / 32];
  const int row = blockIdx.x;
  const int b = row / p.L, t = row - b * p.L;
  const int D = p.D;
  const Row gate_row = param_row(p.gate, b, t);
  float v[CH][8];
#pragma unroll
  for (int j = 0; j < CH; ++j) {
    const int c = (j * NT + threadIdx.x) * 8;
    bf8_to_f32(__ldg(reinterpret_cast<const uint4*>(p.x + b * p.x_bs + t * p.x_rs + c)), v[j]);
  }
  if (p.y) {
#pragma unroll
    for (int j = 0; j < CH; ++j) {
      const int c = (j * NT + threadIdx.x) * 8;
      float y[8];
      bf8_to_f32(__ldg(reinterpret_cast<const uint4*>(p.y + b * p.y_bs + t * p.y_rs + c)), y);
      if (p.gate_idx >= 0) {
        float g[8];
        param8(gate_row, p.gate_idx, D, c, g);
#pragma unroll
        for (int i = 0; i < 8; ++i) y[i] *= g[i];
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) v[j][i] += y[i];
      const uint4 r = f32_to_bf8(v[j]);
      if (p.xo) *reinterpret_cast<uint4*>(p.xo + b * p.xo_bs + t * p.xo_rs + c) = r;
      bf8_to_f32(r, v[j]);  // the norm reads the stored (rounded) residual
    }
  }
  if (p.n_out == 0) return;
  float mean = 0.f;
  if (p.norm_kind == 1) {
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < CH; ++j)
#pragma unroll
      for (int i = 0; i < 8; ++i) s += v[j][i];
    mean = block_sum<NT>(s, red) / static_cast<float>(D);
  }
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < CH; ++j)
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float d = v[j][i] - mean;
      ss += d * d;
    }
  const float inv = rsqrtf(block_sum<NT>(ss, red) / static_cast<float>(D) + p.eps);
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    if (k >= p.n_out) break;
    const Row mod_row = param_row(p.mod[k], b, t);
#pragma unroll
    for (int j = 0; j < CH; ++j) {
      const int c = (j * NT + threadIdx.x) * 8;
      float o[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = (v[j][i] - mean) * inv;
      if (p.scale_idx[k] >= 0) {
        float sc[8], sh[8];
        param8(mod_row, p.scale_idx[k], D, c, sc);
        param8(mod_row, p.shift_idx[k], D, c, sh);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = o[i] * (1.f + sc[i]) + sh[i];
      }
      *reinterpret_cast<uint4*>(p.out[k] + b * p.out_bs[k] + t * p.out_rs[k] + c) =
          f32_to_bf8(o);
    }
  }
}

// gelu(x) = 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))), in place.
__global__ void __launch_bounds__(256) gelu_tanh_kernel(__nv_bfloat16* x, int64_t n_vec) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n_vec;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    uint4* ptr = reinterpret_cast<uint4*>(x) + i;
    float f[8];
    bf8_to_f32(*ptr, f);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float u = f[j];
      f[j] = 0.5f * u * (1.f + tanhf(k0 * (u + k1 * u * u * u)));
    }
    *ptr = f32_to_bf8(f);
  }
}

static int num_sms() {
  static int sms[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!sms[dev]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    sms[dev] = v > 0 ? v : 148;
  }
  return sms[dev];
}

static bool strides_ok(int64_t a, int64_t b) { return a >= 0 && b >= 0 && !(a & 7) && !(b & 7); }

static int check_src(const tm_ada_source* s, int n_rows_needed, const char* what) {
  if (!s) return set_error(TM_ERR_INVALID_ARGUMENT, "residual_norm: %s source missing", what);
  if (!s->table && !s->ts)
    return set_error(TM_ERR_INVALID_ARGUMENT, "residual_norm: %s source has no table and no "
                     "timestep rows", what);
  if ((s->table && !aligned16(s->table)) || (s->ts && !aligned16(s->ts)))
    return set_error(TM_ERR_ALIGNMENT, "residual_norm: %s source not 16-byte aligned", what);
  if (s->ts && (!strides_ok(s->ts_batch_stride, s->ts_row_stride) || s->ts_row_div < 1 ||
                s->ts_row_offset < 0))
    return set_error(TM_ERR_INVALID_ARGUMENT, "residual_norm: %s timestep strides / row map",
                     what);
  (void)n_rows_needed;
  return TM_OK;
}

static Src to_src(const tm_ada_source* s) {
  Src o{};
  if (!s) return o;
  o.table = static_cast<const __nv_bfloat16*>(s->table);
  o.ts = static_cast<const __nv_bfloat16*>(s->ts);
  o.ts_bs = s->ts_batch_stride;
  o.ts_rs = s->ts_row_stride;
  o.ts_div = s->ts_row_div < 1 ? 1 : s->ts_row_div;
  o.ts_off = s->ts_row_offset;
  return o;
}

}  // namespace adaln
}  // namespace tmb

using namespace tmb;

extern "C" int tm_residual_norm(const void* x, int64_t x_batch_stride, int64_t x_row_stride,
                                const void* y, int64_t y_batch_stride, int64_t y_row_stride,
                                const tm_ada_source* gate, int gate_index, void* x_out,
                                int64_t x_out_batch_stride, int64_t x_out_row_stride,
                                const tm_norm_output* outs, int n_outs, int norm_kind, int B,
                                int L, int D, float eps, void* stream) {
  using namespace tmb::adaln;
  if (B < 1 || L < 0 || D < 256 || D > 8192 || (D % 256))
    return set_error(TM_ERR_INVALID_ARGUMENT, "residual_norm: B=%d L=%d D=%d (D a multiple of "
                     "256, at most 8192)", B, L, D);
  if (n_outs < 0 || n_outs > 2 || (n_outs > 0 && !outs) || norm_kind < 0 || norm_kind > 1)
    return set_error(TM_ERR_INVALID_ARGUMENT, "residual_norm: %d outputs, norm kind %d", n_outs,
                     norm_kind);
  if (!x || !aligned16(x) || !strides_ok(x_batch_stride, x_row_stride))
    return set_error(TM_ERR_ALIGNMENT, "residual_norm: x null, unaligned or strides not "
                     "multiples of 8");
  if (y && (!aligned16(y) || !strides_ok(y_batch_stride, y_row_stride)))
    return set_error(TM_ERR_ALIGNMENT, "residual_norm: y unaligned");
  if (y && !x_out && n_outs == 0)
    return set_error(TM_ERR_INVALID_ARGUMENT, "residual_norm: residual sum neither stored nor "
                     "normalised");
  if (x_out && (!y || !aligned16(x_out) || !strides_ok(x_out_batch_stride, x_out_row_stride)))
    return set_error(TM_ERR_INVALID_ARGUMENT, "residual_norm: x_out needs y and 16-byte "
                     "alignment");
  if (x_row_stride < D || (y && y_row_stride < D) || (x_out && x_out_row_stride < D))
    return set_error(TM_ERR_INVALID_ARGUMENT, "residual_norm: row stride below D");
  Params p;
  memset(&p, 0, sizeof(p));
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.x_bs = B > 1 ? x_batch_stride : 0;
  p.x_rs = x_row_stride;
  p.y = static_cast<const __nv_bfloat16*>(y);
  p.y_bs = B > 1 ? y_batch_stride : 0;
  p.y_rs = y_row_stride;
  p.xo = static_cast<__nv_bfloat16*>(x_out);
  p.xo_bs = B > 1 ? x_out_batch_stride : 0;
  p.xo_rs = x_out_row_stride;
  p.gate_idx = -1;
  if (y && gate && gate_index >= 0) {
    const int st = check_src(gate, gate_index + 1, "gate");
    if (st) return st;
    p.gate = to_src(gate);
    p.gate_idx = gate_index;
  }
  p.n_out = n_outs;
  for (int k = 0; k < n_outs; ++k) {
    const tm_norm_output& o = outs[k];
    if (!o.out || !aligned16(o.out) || !strides_ok(o.batch_stride, o.row_stride) ||
        o.row_stride < D)
      return set_error(TM_ERR_ALIGNMENT, "residual_norm: output %d null, unaligned or bad "
                       "strides", k);
    p.out[k] = static_cast<__nv_bfloat16*>(o.out);
    p.out_bs[k] = B > 1 ? o.batch_stride : 0;
    p.out_rs[k] = o.row_stride;
    p.scale_idx[k] = o.scale_index;
    p.shift_idx[k] = o.shift_index;
    if (o.scale_index >= 0) {
      if (o.shift_index < 0)
        return set_error(TM_ERR_INVALID_ARGUMENT, "residual_norm: output %d has a scale but no "
                         "shift", k);
      const int st = check_src(&o.mod, 1, "modulation");
      if (st) return st;
      p.mod[k] = to_src(&o.mod);
    }
  }
  p.norm_kind = norm_kind;
  p.L = L;
  p.D = D;
  p.eps = eps;
  if (L == 0) return TM_OK;
  const int64_t rows = static_cast<int64_t>(B) * L;
  if (rows > 0x7fffffff) return set_error(TM_ERR_INVALID_ARGUMENT, "residual_norm: too many rows");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid(static_cast<unsigned>(rows));
  switch (D / 8) {  // threads x chunks
    case 32: residual_norm_kernel<32, 1><<<grid, 32, 0, s>>>(p); break;
    case 64: residual_norm_kernel<64, 1><<<grid, 64, 0, s>>>(p); break;
    case 96: residual_norm_kernel<96, 1><<<grid, 96, 0, s>>>(p); break;
    case 128: residual_norm_kernel<128, 1><<<grid, 128, 0, s>>>(p); break;
    case 160: residual_norm_kernel<160, 1><<<grid, 160, 0, s>>>(p); break;
    case 192: residual_norm_kernel<192, 1><<<grid, 192, 0, s>>>(p); break;
    case 224: residual_norm_kernel<224, 1><<<grid, 224, 0, s>>>(p); break;
    case 256: residual_norm_kernel<256, 1><<<grid, 256, 0, s>>>(p); break;
    case 384: residual_norm_kernel<192, 2><<<grid, 192, 0, s>>>(p); break;
    case 512: residual_norm_kernel<256, 2><<<grid, 256, 0, s>>>(p); break;
    case 768: residual_norm_kernel<192, 4><<<grid, 192, 0, s>>>(p); break;
    case 1024: residual_norm_kernel<256, 4><<<grid, 256, 0, s>>>(p); break;
    default:
      return set_error(TM_ERR_UNSUPPORTED, "residual_norm: D=%d not built", D);
  }
  return check_cuda(cudaGetLastError(), "residual_norm: launch");
}

extern "C" int tm_gelu_tanh(void* x, int64_t n, void* stream) {
  using namespace tmb::adaln;
  if (n < 0 || (n & 7)) return set_error(TM_ERR_INVALID_ARGUMENT, "gelu: %lld elements (a "
                                         "multiple of 8)", (long long)n);
  if (n == 0) return TM_OK;
  if (!x || !aligned16(x)) return set_error(TM_ERR_ALIGNMENT, "gelu: x null or unaligned");
  const int64_t nv = n / 8;
  const int64_t per = static_cast<int64_t>(num_sms()) * 8 * 256;
  const int blocks = static_cast<int>(std::min<int64_t>((nv + 255) / 256, per / 256));
  gelu_tanh_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<__nv_bfloat16*>(x), nv);
  return check_cuda(cudaGetLastError(), "gelu: launch");
}
