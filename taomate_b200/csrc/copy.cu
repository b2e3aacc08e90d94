// Copy kernels for the KV slot arena (append / compaction / materialise) and
// the layout permutes around the Ulysses all-to-all.  Both move 16-byte
// vectors with consecutive threads on consecutive addresses of a row, so
// reads and writes are fully coalesced; grids are sized in multiples of the
// SM count.
#include <algorithm>

#include "common.cuh"
#include "host_common.h"

namespace tmb {
namespace copy {

constexpr int kMaxSpans = 64;

struct Span {
  const uint8_t* src;
  uint8_t* dst;
  int64_t rows, srs, drs;
};

struct RowsParams {
  Span spans[kMaxSpans];
  int n;
  int64_t vec_per_row;  // row_bytes / 16
};

// Each thread keeps kBatch independent 16-byte loads in flight before it
// stores them (the loads of one batch index are coalesced across the warp);
// a grid of about one wave then streams at HBM speed.  Index arithmetic in
// 32 bits (a span's vectors are checked to fit on the host).
constexpr int kBatch = 4;

__global__ void __launch_bounds__(256) copy_rows_kernel(const __grid_constant__ RowsParams p) {
  const Span& s = p.spans[blockIdx.y];
  const uint32_t total = static_cast<uint32_t>(s.rows * p.vec_per_row);
  const uint32_t vpr = static_cast<uint32_t>(p.vec_per_row);
  const uint32_t stride = gridDim.x * blockDim.x;
  for (uint32_t base = blockIdx.x * blockDim.x + threadIdx.x; base < total;
       base += kBatch * stride) {
    uint4 x[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const uint32_t i = base + u * stride;
      if (i < total) {
        const uint32_t r = i / vpr, v = i - r * vpr;
        x[u] = __ldg(reinterpret_cast<const uint4*>(s.src + static_cast<int64_t>(r) * s.srs) + v);
      }
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const uint32_t i = base + u * stride;
      if (i < total) {
        const uint32_t r = i / vpr, v = i - r * vpr;
        *(reinterpret_cast<uint4*>(s.dst + static_cast<int64_t>(r) * s.drs) + v) = x[u];
      }
    }
  }
}

struct Strided5 {
  const uint8_t* src;
  uint8_t* dst;
  int64_t size[4];  // outer sizes
  int64_t sst[4];   // byte strides of the outer dims
  int64_t dst_[4];
  int64_t vec;      // 16-byte vectors in the contiguous innermost dim
  int64_t total;
};

__global__ void __launch_bounds__(256) strided5_kernel(const __grid_constant__ Strided5 p) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < p.total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t rem = i / p.vec;
    const int64_t v = i - rem * p.vec;
    int64_t so = 0, dof = 0;
#pragma unroll
    for (int d = 3; d >= 0; --d) {
      const int64_t idx = rem % p.size[d];
      rem /= p.size[d];
      so += idx * p.sst[d];
      dof += idx * p.dst_[d];
    }
    const uint4 x = __ldg(reinterpret_cast<const uint4*>(p.src + so) + v);
    *(reinterpret_cast<uint4*>(p.dst + dof) + v) = x;
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

}  // namespace copy
}  // namespace tmb

using namespace tmb;

extern "C" int tm_copy_rows(const tm_copy_span* spans, int n_spans, int64_t row_bytes,
                            void* stream) {
  using namespace tmb::copy;
  if (!spans || n_spans < 1 || n_spans > kMaxSpans)
    return set_error(TM_ERR_INVALID_ARGUMENT, "copy_rows: %d spans (1..%d)", n_spans, kMaxSpans);
  if (row_bytes <= 0 || (row_bytes & 15))
    return set_error(TM_ERR_ALIGNMENT, "copy_rows: row_bytes %lld not a multiple of 16",
                     (long long)row_bytes);
  RowsParams p;
  memset(&p, 0, sizeof(p));
  p.n = n_spans;
  p.vec_per_row = row_bytes / 16;
  int64_t max_units = 0;
  for (int i = 0; i < n_spans; ++i) {
    const tm_copy_span& s = spans[i];
    if (s.rows < 0) return set_error(TM_ERR_INVALID_ARGUMENT, "copy_rows: span %d rows < 0", i);
    if (s.rows > 0 && (!s.src || !s.dst))
      return set_error(TM_ERR_INVALID_ARGUMENT, "copy_rows: span %d null pointer", i);
    if (!aligned16(s.src) || !aligned16(s.dst) || (s.src_row_stride & 15) ||
        (s.dst_row_stride & 15))
      return set_error(TM_ERR_ALIGNMENT, "copy_rows: span %d not 16-byte aligned", i);
    p.spans[i].src = static_cast<const uint8_t*>(s.src);
    p.spans[i].dst = static_cast<uint8_t*>(s.dst);
    p.spans[i].rows = s.rows;
    p.spans[i].srs = s.src_row_stride;
    p.spans[i].drs = s.dst_row_stride;
    const int64_t u = s.rows * p.vec_per_row;
    if (u >= (int64_t(1) << 31))
      return set_error(TM_ERR_INVALID_ARGUMENT, "copy_rows: span %d has 2^31 or more 16-byte "
                       "vectors", i);
    if (u > max_units) max_units = u;
  }
  if (max_units == 0) return TM_OK;
  const int threads = 256;
  int64_t bx = (max_units + threads * kBatch - 1) / (threads * kBatch);
  // about one wave of 8 blocks per SM over all spans
  const int64_t cap = std::max<int64_t>(1, static_cast<int64_t>(num_sms()) * 8 / n_spans);
  if (bx > cap) bx = cap;
  dim3 grid(static_cast<unsigned>(bx), static_cast<unsigned>(n_spans));
  copy_rows_kernel<<<grid, threads, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return check_cuda(cudaGetLastError(), "copy_rows: launch");
}

extern "C" int tm_strided_copy5(const void* src, void* dst, const int64_t* sizes,
                                const int64_t* src_strides, const int64_t* dst_strides,
                                int elem_bytes, void* stream) {
  using namespace tmb::copy;
  if (!src || !dst || !sizes || !src_strides || !dst_strides || elem_bytes <= 0)
    return set_error(TM_ERR_INVALID_ARGUMENT, "strided_copy5: null argument");
  const int64_t inner_bytes = sizes[4] * elem_bytes;
  if (sizes[4] < 1 || (inner_bytes & 15))
    return set_error(TM_ERR_ALIGNMENT, "strided_copy5: inner extent %lld bytes not a multiple of 16",
                     (long long)inner_bytes);
  if (!aligned16(src) || !aligned16(dst))
    return set_error(TM_ERR_ALIGNMENT, "strided_copy5: pointer not 16-byte aligned");
  Strided5 p;
  memset(&p, 0, sizeof(p));
  p.src = static_cast<const uint8_t*>(src);
  p.dst = static_cast<uint8_t*>(dst);
  int64_t outer = 1;
  for (int d = 0; d < 4; ++d) {
    if (sizes[d] < 1) return TM_OK;
    const int64_t sb = src_strides[d] * elem_bytes, db = dst_strides[d] * elem_bytes;
    if ((sb & 15) || (db & 15))
      return set_error(TM_ERR_ALIGNMENT, "strided_copy5: dim %d stride not 16-byte aligned", d);
    p.size[d] = sizes[d];
    p.sst[d] = sb;
    p.dst_[d] = db;
    outer *= sizes[d];
  }
  if (src_strides[4] != 1 || dst_strides[4] != 1)
    return set_error(TM_ERR_INVALID_ARGUMENT, "strided_copy5: innermost dim must be contiguous");
  p.vec = inner_bytes / 16;
  p.total = outer * p.vec;
  const int threads = 256;
  int64_t blocks = (p.total + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(num_sms()) * 8;
  if (blocks > cap) blocks = cap;
  strided5_kernel<<<static_cast<unsigned>(blocks), threads, 0, static_cast<cudaStream_t>(stream)>>>(
      p);
  return check_cuda(cudaGetLastError(), "strided_copy5: launch");
}
