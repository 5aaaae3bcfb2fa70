// Segment engine kernels: centred zero-padded chunk gather, triangular
// weighted overlap-add with a weight sum, in-place weighting of trimmed chunk
// outputs (for accumulation on the host), and the final divide
// (unblend/apply.py:278-311 TensorChunk.padded, 406-432 _split_weight,
// 1219-1238 accumulate, 1329 out / sum_weight). HBM-streaming, fp32.
#include "common.cuh"

namespace {

// Triangular cross-fade weight of unblend/apply.py:426-430: rising 1..half,
// falling (T-half)..1, divided by the max, raised to the transition power
// (the fp32 quotient first, then powf, as the reference's fp32 tensor ops).
__device__ __forceinline__ float split_weight(int j, int seg, float power) {
  const int half = seg / 2;
  const float mx = (float)(half > seg - half ? half : seg - half);
  const float v = j < half ? (float)(j + 1) : (float)(seg - j);
  const float w = v / mx;
  return power == 1.f ? w : powf(w, power);
}

__global__ void gather_chunks_kernel(const float* __restrict__ track, int channels, long long length,
                                     const long long* __restrict__ offsets, int n, int seg,
                                     float* __restrict__ batch) {
  const long long total = (long long)n * channels * seg;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int j = (int)(i % seg);
    const long long ic = i / seg;
    const int c = (int)(ic % channels);
    const int k = (int)(ic / channels);
    const long long o = offsets[k];
    const long long len = length - o < seg ? length - o : seg;
    const long long start = o - (seg - len) / 2;
    const long long src = start + j;
    batch[i] = (src >= 0 && src < length) ? __ldg(track + (long long)c * length + src) : 0.f;
  }
}

// acc[r, p] += w(j) y[k, r, trim_k + j] and sum_w[p] += w(j) over the chunks k holding p, in
// chunk order, each product rounded before its addition: the per-chunk accumulation of
// unblend/apply.py:1214-1238 in the same order, so the result does not depend on how the
// chunks were split into batches.
__global__ void overlap_add_kernel(const float* __restrict__ y, int n, int rows, int seg,
                                   const long long* __restrict__ offsets, long long length, long long lo,
                                   long long span, float power, float* __restrict__ acc,
                                   float* __restrict__ sum_w) {
  const long long total = (long long)rows * span;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long p = lo + i % span;
    const int r = (int)(i / span);
    if (p >= length) continue;
    // Offsets ascend, so the chunks holding p start in (p - seg, p]: find the
    // first with offset > p - seg by bisection (a position lies in at most
    // ceil(seg / stride) chunks) instead of testing all n.
    int k0 = 0, k1 = n;
    while (k0 < k1) {
      const int mid = (k0 + k1) >> 1;
      if (__ldg(offsets + mid) > p - seg) k1 = mid;
      else k0 = mid + 1;
    }
    float a = acc[(long long)r * length + p], ws = r == 0 ? sum_w[p] : 0.f;
    for (int k = k0; k < n; ++k) {
      const long long o = __ldg(offsets + k);
      if (o > p) break;
      const long long len = length - o < seg ? length - o : seg;
      const long long j = p - o;
      if (j >= len) continue;
      const int trim = (int)((seg - len) / 2);
      const float w = split_weight((int)j, seg, power);
      a = __fadd_rn(a, __fmul_rn(w, y[((long long)k * rows + r) * seg + trim + j]));
      ws = __fadd_rn(ws, w);
    }
    acc[(long long)r * length + p] = a;
    if (r == 0) sum_w[p] = ws;
  }
}

// y[k, r, trim_k + j] *= w(j) for j < len_k (the chunk's valid length): the
// contribution of chunk k before it is added on the host.
__global__ void weight_chunks_kernel(float* __restrict__ y, int n, int rows, int seg,
                                     const long long* __restrict__ offsets, long long length, float power) {
  const long long total = (long long)n * rows * seg;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int t = (int)(i % seg);
    const int k = (int)(i / ((long long)rows * seg));
    const long long o = __ldg(offsets + k);
    const int len = (int)(length - o < seg ? length - o : seg);
    const int trim = (seg - len) / 2;
    const int j = t - trim;
    if (j >= 0 && j < len) y[i] *= split_weight(j, seg, power);
  }
}

__global__ void divide_kernel(const float* __restrict__ acc, const float* __restrict__ sum_w,
                              float* __restrict__ out, int rows, long long length) {
  const long long total = (long long)rows * length;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x)
    out[i] = acc[i] / sum_w[i % length];
}

}  // namespace

extern "C" int unblend_gather_chunks(const float* track, int channels, long long length, const long long* offsets,
                                     int n, int segment, float* batch, void* stream) {
  UB_REQUIRE(track && offsets && batch && channels > 0 && length > 0 && n > 0 && segment > 0);
  const long long total = (long long)n * channels * segment;
  gather_chunks_kernel<<<ub::grid_1d(total, 256), 256, 0, ub::as_stream(stream)>>>(
      track, channels, length, offsets, n, segment, batch);
  UB_CHECK_LAUNCH();
  return 0;
}

// offsets: n chunk starts in ascending order.
extern "C" int unblend_overlap_add(const float* y, int n, int rows, int segment, const long long* offsets,
                                   long long length, long long lo, long long hi, float power, float* acc,
                                   float* sum_w, void* stream) {
  UB_REQUIRE(y && offsets && acc && sum_w && n > 0 && rows > 0 && segment > 0 && length > 0);
  UB_REQUIRE(lo >= 0 && hi > lo && power > 0.f);
  const long long span = hi - lo;
  overlap_add_kernel<<<ub::grid_1d((long long)rows * span, 256), 256, 0, ub::as_stream(stream)>>>(
      y, n, rows, segment, offsets, length, lo, span, power, acc, sum_w);
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_weight_chunks(float* y, int n, int rows, int segment, const long long* offsets,
                                     long long length, float power, void* stream) {
  UB_REQUIRE(y && offsets && n > 0 && rows > 0 && segment > 0 && length > 0 && power > 0.f);
  const long long total = (long long)n * rows * segment;
  weight_chunks_kernel<<<ub::grid_1d(total, 256), 256, 0, ub::as_stream(stream)>>>(
      y, n, rows, segment, offsets, length, power);
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_divide(const float* acc, const float* sum_w, float* out, int rows, long long length,
                              void* stream) {
  UB_REQUIRE(acc && sum_w && out && rows > 0 && length > 0);
  divide_kernel<<<ub::grid_1d((long long)rows * length, 256), 256, 0, ub::as_stream(stream)>>>(
      acc, sum_w, out, rows, length);
  UB_CHECK_LAUNCH();
  return 0;
}
