// Multi-head attention core, fp32 SIMT flash-attention (online softmax).
//
// Computes softmax(Q K^T * scale) V per (batch, head) exactly as
// nn.MultiheadAttention does in eval mode without masks
// (unblend/transformer.py:290-301 self-attention, 402-412 cross-attention),
// without materialising the Lq x Lk score matrix. One CTA owns 64 queries of
// one head and streams K/V in tiles of 64 keys through shared memory.
#include "common.cuh"

namespace {

constexpr int BQ = 64;
constexpr int BKV = 64;
constexpr int HD = 64;  // head dim padded to 64 in shared memory
constexpr int NT = 128;

struct AttnArgs {
  const float* q;
  const float* k;
  const float* v;
  float* o;
  int heads, lq, lk, hd;
  long long q_sb, q_sr, kv_sb, kv_sr, o_sb, o_sr;
  float scale;
};

__global__ void __launch_bounds__(NT) attention_simt_kernel(AttnArgs a) {
  extern __shared__ __align__(16) float smem[];
  float* Qs = smem;                  // [HD][BQ]   (d-major)
  float* Ks = Qs + HD * BQ;          // [HD][BKV]  (d-major)
  float* Vs = Ks + HD * BKV;         // [BKV][HD]
  float* Ps = Vs + BKV * HD;         // [BKV][BQ]  (key-major)

  const int tid = threadIdx.x;
  const int tx = tid & 15;  // 16 lanes across keys (S) or dims (O)
  const int ty = tid >> 4;  // 8 groups of 8 query rows
  const int qblk = blockIdx.x;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int q0 = qblk * BQ;

  const float* qb = a.q + (long long)b * a.q_sb + (long long)h * a.hd;
  const float* kb = a.k + (long long)b * a.kv_sb + (long long)h * a.hd;
  const float* vb = a.v + (long long)b * a.kv_sb + (long long)h * a.hd;

  // Load Q tile (scaled), transposed to d-major.
  for (int idx = tid; idx < BQ * HD; idx += NT) {
    int r = idx / HD, d = idx - r * HD;
    float val = 0.f;
    if (q0 + r < a.lq && d < a.hd) val = qb[(long long)(q0 + r) * a.q_sr + d] * a.scale;
    Qs[d * BQ + r] = val;
  }

  float o[8][4];
  float mrow[8], lrow[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    mrow[i] = -INFINITY;
    lrow[i] = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) o[i][j] = 0.f;
  }

  for (int k0 = 0; k0 < a.lk; k0 += BKV) {
    __syncthreads();
    for (int idx = tid; idx < BKV * HD; idx += NT) {
      int r = idx / HD, d = idx - r * HD;
      float kv = 0.f, vv = 0.f;
      if (k0 + r < a.lk && d < a.hd) {
        kv = kb[(long long)(k0 + r) * a.kv_sr + d];
        vv = vb[(long long)(k0 + r) * a.kv_sr + d];
      }
      Ks[d * BKV + r] = kv;
      Vs[r * HD + d] = vv;
    }
    __syncthreads();

    // S = Q K^T for rows ty*8..+8, keys tx*4..+4.
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.f;
    for (int d = 0; d < HD; ++d) {
      float4 qa = *reinterpret_cast<const float4*>(Qs + d * BQ + ty * 8);
      float4 qc = *reinterpret_cast<const float4*>(Qs + d * BQ + ty * 8 + 4);
      float4 kk = *reinterpret_cast<const float4*>(Ks + d * BKV + tx * 4);
      float qv[8] = {qa.x, qa.y, qa.z, qa.w, qc.x, qc.y, qc.z, qc.w};
      float kv[4] = {kk.x, kk.y, kk.z, kk.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) s[i][j] = fmaf(qv[i], kv[j], s[i][j]);
    }
    // Online softmax update per row (16 lanes share a row).
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (k0 + tx * 4 + j >= a.lk) s[i][j] = -INFINITY;
        mx = fmaxf(mx, s[i][j]);
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      float mnew = fmaxf(mrow[i], mx);
      float corr = expf(mrow[i] - mnew);
      float ps = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float pv = expf(s[i][j] - mnew);
        s[i][j] = pv;
        ps += pv;
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
      lrow[i] = lrow[i] * corr + ps;
      mrow[i] = mnew;
#pragma unroll
      for (int j = 0; j < 4; ++j) o[i][j] *= corr;
    }
    // Stage P (key-major) for the PV product.
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) Ps[(tx * 4 + j) * BQ + ty * 8 + i] = s[i][j];
    __syncthreads();
    // O[rows, dims tx*4..+4] += P V.
    for (int j = 0; j < BKV; ++j) {
      float4 pa = *reinterpret_cast<const float4*>(Ps + j * BQ + ty * 8);
      float4 pc = *reinterpret_cast<const float4*>(Ps + j * BQ + ty * 8 + 4);
      float4 vv = *reinterpret_cast<const float4*>(Vs + j * HD + tx * 4);
      float pv[8] = {pa.x, pa.y, pa.z, pa.w, pc.x, pc.y, pc.z, pc.w};
      float vr[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int d = 0; d < 4; ++d) o[i][d] = fmaf(pv[i], vr[d], o[i][d]);
    }
  }

  float* ob = a.o + (long long)b * a.o_sb + (long long)h * a.hd;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int r = q0 + ty * 8 + i;
    if (r >= a.lq) continue;
    float inv = 1.f / lrow[i];
#pragma unroll
    for (int d = 0; d < 4; ++d) {
      int dd = tx * 4 + d;
      if (dd < a.hd) ob[(long long)r * a.o_sr + dd] = o[i][d] * inv;
    }
  }
}

}  // namespace

extern "C" int unblend_attention_f32(const float* q, const float* k, const float* v, float* out, int batch,
                                     int heads, int lq, int lk, int hd, long long q_sb, long long q_sr,
                                     long long kv_sb, long long kv_sr, long long o_sb, long long o_sr,
                                     float scale, void* stream) {
  UB_REQUIRE(q && k && v && out && batch > 0 && heads > 0 && lq > 0 && lk > 0);
  UB_REQUIRE(hd > 0 && hd <= HD && heads < 65536 && batch < 65536);
  AttnArgs a{q, k, v, out, heads, lq, lk, hd, q_sb, q_sr, kv_sb, kv_sr, o_sb, o_sr, scale};
  size_t smem = sizeof(float) * (HD * BQ + HD * BKV + BKV * HD + BKV * BQ);
  cudaFuncSetAttribute(attention_simt_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid((lq + BQ - 1) / BQ, heads, batch);
  attention_simt_kernel<<<grid, NT, smem, ub::as_stream(stream)>>>(a);
  UB_CHECK_LAUNCH();
  return 0;
}
