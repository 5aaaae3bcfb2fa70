// Band gather and scatter-average of the Mel-Band RoFormer (fp32).
//
// The mel bands overlap, so BandSplit reads each band's bins through an index
// list and the mask estimators' per-band outputs are summed back onto the bins
// and divided by the number of bands covering each bin
// (unblend/roformer.py:1541-1575: index_select, scatter_add_, divide). Both
// move (re, im) pairs: element pair j of a row is floats 2j, 2j+1.
#include "common.cuh"

namespace {

// dst[r, j] = src[r, idx[j]] (pairs), one thread per (row, j) with j fastest.
__global__ void gather_pairs_kernel(const float2* __restrict__ src, long long src_ld2, long long rows,
                                    const int* __restrict__ idx, int n, float2* __restrict__ dst, long long dst_ld2) {
  const long long total = rows * n;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / n;
    const int j = (int)(i - r * n);
    dst[r * dst_ld2 + j] = __ldg(src + r * src_ld2 + __ldg(idx + j));
  }
}

// dst[r, c] = sum over q in [off[c], off[c+1]) of src[r, pos[q]] / count (pairs),
// summed in ascending q.
__global__ void scatter_mean_pairs_kernel(const float2* __restrict__ src, long long src_ld2, long long rows,
                                          const int* __restrict__ off, const int* __restrict__ pos, int n_dst,
                                          float2* __restrict__ dst, long long dst_ld2) {
  const long long total = rows * n_dst;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / n_dst;
    const int c = (int)(i - r * n_dst);
    const int q0 = __ldg(off + c), q1 = __ldg(off + c + 1);
    const float2* row = src + r * src_ld2;
    float sx = 0.f, sy = 0.f;
    for (int q = q0; q < q1; ++q) {
      const float2 v = __ldg(row + __ldg(pos + q));
      sx += v.x;
      sy += v.y;
    }
    const float cnt = (float)(q1 - q0);
    dst[r * dst_ld2 + c] = q1 > q0 ? make_float2(sx / cnt, sy / cnt) : make_float2(0.f, 0.f);
  }
}

}  // namespace

extern "C" int unblend_gather_pairs(const float* src, long long src_ld, long long rows, const int* idx, int n,
                                    float* dst, long long dst_ld, void* stream) {
  UB_REQUIRE(src && idx && dst && rows > 0 && n > 0 && src_ld % 2 == 0 && dst_ld % 2 == 0 && dst_ld >= 2LL * n);
  UB_REQUIRE((reinterpret_cast<uintptr_t>(src) & 7) == 0 && (reinterpret_cast<uintptr_t>(dst) & 7) == 0);
  gather_pairs_kernel<<<ub::grid_1d(rows * n, 256), 256, 0, ub::as_stream(stream)>>>(
      reinterpret_cast<const float2*>(src), src_ld / 2, rows, idx, n, reinterpret_cast<float2*>(dst), dst_ld / 2);
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_scatter_mean_pairs(const float* src, long long src_ld, long long rows, const int* offsets,
                                          const int* pos, int n_dst, float* dst, long long dst_ld, void* stream) {
  UB_REQUIRE(src && offsets && pos && dst && rows > 0 && n_dst > 0 && src_ld % 2 == 0 && dst_ld % 2 == 0 &&
             dst_ld >= 2LL * n_dst);
  UB_REQUIRE((reinterpret_cast<uintptr_t>(src) & 7) == 0 && (reinterpret_cast<uintptr_t>(dst) & 7) == 0);
  scatter_mean_pairs_kernel<<<ub::grid_1d(rows * n_dst, 256), 256, 0, ub::as_stream(stream)>>>(
      reinterpret_cast<const float2*>(src), src_ld / 2, rows, offsets, pos, n_dst, reinterpret_cast<float2*>(dst),
      dst_ld / 2);
  UB_CHECK_LAUNCH();
  return 0;
}
