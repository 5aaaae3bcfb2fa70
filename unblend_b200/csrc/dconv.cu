// Fused DConv residual branch (unblend/blocks.py:238-317), fp32, HBM-streaming.
//
// One DConv layer is  x += LayerScale * GLU(GN2(W2 * GELU(GN1(conv_k3_dil(x)))))
// with GroupNorm(1) statistics per group (a (batch, frequency) row of the
// frequency branch, or a batch item of the time branch). The hidden width is
// C/8, so both contractions are far too thin for tensor cores to pay; the
// cost is moving x. The kernels:
//   dconv_conv1        h = conv_k3_dil(x) with GN1 sums (x rows + weights in smem;
//                      conv1b: register-blocked, every hidden output of 3 rows per lane)
//   dconv_moments      a = GELU(GN1(h)) written over h, with the sums of a and of
//                      a a^T per group
//   dconv_moment_sums  GN2 statistics of z = W2 a + b2 from those moments and the
//                      float64 coefficients W2^T 1, W2^T b2, W2^T W2 (z never exists)
//   dconv_apply        recompute z from a, x += scale * GLU(GN2(z)) in place
// x element (g, r, c) is at x + g * x_gs + r * C + c; h is contiguous
// [groups, rows, H]. W1 is [H, 3, C]; W2 is [2C, H] with rows interleaved as
// (value 0, gate 0, value 1, gate 1, ...), GN2 affine in the same order.
#include "common.cuh"

namespace {

constexpr int ROWS = 128;  // rows per CTA, one thread per row

template <int MAXH>
__global__ void __launch_bounds__(ROWS) dconv_conv1_kernel(const float* __restrict__ x, long long x_gs, int rows,
                                                           int C, const float* __restrict__ w1,
                                                           const float* __restrict__ b1, int H, int dil,
                                                           float* __restrict__ h, double* __restrict__ stats) {
  extern __shared__ __align__(16) float sm[];
  const int CP = C + 4;  // padded row stride (keeps 16-byte alignment)
  float* xs = sm;                                  // [ROWS + 2*dil][CP]
  float* ws = sm + (ROWS + 2 * dil) * CP;          // [H][3][C]
  const int g = blockIdx.y;
  const int r0 = blockIdx.x * ROWS;
  const float* xg = x + (long long)g * x_gs;
  const int nrows = ROWS + 2 * dil;
  // Stage the x rows [r0 - dil, r0 + ROWS + dil) (zero outside [0, rows)).
  const int c4 = C / 4;
  for (int i = threadIdx.x; i < nrows * c4; i += ROWS) {
    const int rr = i / c4, cc = (i - rr * c4) * 4;
    const int r = r0 - dil + rr;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r >= 0 && r < rows) v = *reinterpret_cast<const float4*>(xg + (long long)r * C + cc);
    *reinterpret_cast<float4*>(xs + rr * CP + cc) = v;
  }
  for (int i = threadIdx.x; i < H * 3 * C; i += ROWS) ws[i] = w1[i];
  __syncthreads();
  const int lr = threadIdx.x;
  const int r = r0 + lr;
  float acc[MAXH];
#pragma unroll
  for (int j = 0; j < MAXH; ++j) acc[j] = (j < H) ? __ldg(b1 + j) : 0.f;
  for (int t = 0; t < 3; ++t) {
    const float* xr = xs + (lr + t * dil) * CP;
    for (int c = 0; c < C; c += 4) {
      const float4 xv = *reinterpret_cast<const float4*>(xr + c);
#pragma unroll
      for (int j = 0; j < MAXH; ++j) {
        if (j < H) {
          const float4 wv = *reinterpret_cast<const float4*>(ws + (j * 3 + t) * C + c);
          acc[j] = fmaf(xv.x, wv.x, fmaf(xv.y, wv.y, fmaf(xv.z, wv.z, fmaf(xv.w, wv.w, acc[j]))));
        }
      }
    }
  }
  float s1 = 0.f, s2 = 0.f;
  if (r < rows) {
    float* hr = h + ((long long)g * rows + r) * H;
#pragma unroll
    for (int j = 0; j < MAXH; ++j) {
      if (j < H) {
        hr[j] = acc[j];
        s1 += acc[j];
        s2 += acc[j] * acc[j];
      }
    }
  }
  s1 = ub::warp_sum(s1);
  s2 = ub::warp_sum(s2);
  __shared__ float red[2][ROWS / 32];
  if ((threadIdx.x & 31) == 0) {
    red[0][threadIdx.x >> 5] = s1;
    red[1][threadIdx.x >> 5] = s2;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double a = 0, b = 0;
    for (int i = 0; i < ROWS / 32; ++i) {
      a += red[0][i];
      b += red[1][i];
    }
    atomicAdd(stats + 2 * g, a);
    atomicAdd(stats + 2 * g + 1, b);
  }
}

// GELU(GN1(h)) of one row into registers.
template <int MAXH>
__device__ __forceinline__ void load_act(const float* __restrict__ hr, int H, float mean, float rstd,
                                         const float* __restrict__ g1w, const float* __restrict__ g1b,
                                         float (&a)[MAXH]) {
#pragma unroll
  for (int j = 0; j < MAXH; ++j) {
    float v = 0.f;
    if (j < H) v = ub::gelu_erf((hr[j] - mean) * rstd * __ldg(g1w + j) + __ldg(g1b + j));
    a[j] = v;
  }
}

template <int MAXH>
__device__ __forceinline__ float dot_row(const float* __restrict__ wrow, const float (&a)[MAXH], int H, float b) {
  float z = b;
#pragma unroll
  for (int j = 0; j < MAXH; ++j)
    if (j < H) z = fmaf(wrow[j], a[j], z);
  return z;
}

template <int MAXH>
__global__ void __launch_bounds__(ROWS) dconv_apply_kernel(float* __restrict__ x, long long x_gs,
                                                           const float* __restrict__ h, int rows, int H, int C,
                                                           const float* __restrict__ st1,
                                                           const float* __restrict__ g1w,
                                                           const float* __restrict__ g1b,
                                                           const float* __restrict__ w2,
                                                           const float* __restrict__ b2,
                                                           const float* __restrict__ st2,
                                                           const float* __restrict__ g2w,
                                                           const float* __restrict__ g2b,
                                                           const float* __restrict__ scale) {
  extern __shared__ __align__(16) float sm[];
  float* ws = sm;             // [2C][H]
  float* bs = ws + 2 * C * H; // [2C]
  float* gw = bs + 2 * C;     // [2C] GN2 gamma * rstd
  float* gb = gw + 2 * C;     // [2C] GN2 beta - mean * rstd * gamma
  float* sc = gb + 2 * C;     // [C]
  const int g = blockIdx.y;
  const float mean2 = st2[2 * g], rstd2 = st2[2 * g + 1];
  for (int i = threadIdx.x; i < 2 * C * H; i += ROWS) ws[i] = w2[i];
  for (int i = threadIdx.x; i < 2 * C; i += ROWS) {
    bs[i] = b2[i];
    gw[i] = g2w[i];
    gb[i] = g2b[i];
  }
  for (int i = threadIdx.x; i < C; i += ROWS) sc[i] = scale[i];
  __syncthreads();
  const int r = blockIdx.x * ROWS + threadIdx.x;
  if (r >= rows) return;
  float a[MAXH];
  load_act<MAXH>(h + ((long long)g * rows + r) * H, H, st1[2 * g], st1[2 * g + 1], g1w, g1b, a);
  float* xr = x + (long long)g * x_gs + (long long)r * C;
  for (int c = 0; c < C; c += 4) {
    float4 xv = *reinterpret_cast<float4*>(xr + c);
    float o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int n = 2 * (c + e);
      const float zv = dot_row<MAXH>(ws + n * H, a, H, bs[n]);
      const float zg = dot_row<MAXH>(ws + (n + 1) * H, a, H, bs[n + 1]);
      const float v = (zv - mean2) * rstd2 * gw[n] + gb[n];
      const float gt = (zg - mean2) * rstd2 * gw[n + 1] + gb[n + 1];
      o[e] = sc[c + e] * (v * ub::sigmoid_approx(gt));
    }
    xv.x += o[0];
    xv.y += o[1];
    xv.z += o[2];
    xv.w += o[3];
    *reinterpret_cast<float4*>(xr + c) = xv;
  }
}

// ---------------------------------------------------------------------------
// Persistent, channel-blocked passes over the thin DConv levels (hidden width
// <= 16, padded to a multiple of 4 by the caller so h rows are 16-byte
// aligned). A CTA walks work items (group, block of IROWS rows) in a
// grid-stride loop with the rows of the next NBUF-1 items already in flight
// (bulk async copies into a shared-memory ring). Thread t keeps the W2 rows of
// its CPT output channels (value and gate rows) in registers for the whole
// kernel and walks rows t / CG, t / CG + RPP, ... of each item; the item's
// activations a = GELU(GN1(h)) sit in shared memory (a broadcast read feeding
// 2*CPT dot products).
constexpr int CPT = 2;      // output channels per thread
constexpr int NTH2 = 256;   // threads per CTA (CG * RPP <= NTH2)

__device__ __forceinline__ uint32_t sm_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

// Bounded wait (about 2 s of %globaltimer) for the phase `parity` of `bar`; false on timeout.
__device__ __forceinline__ bool wait_phase(uint64_t* bar, uint32_t parity) {
  uint64_t t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  while (true) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(sm_u32(bar)), "r"(parity)
        : "memory");
    if (ok) return true;
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (t - t0 > 2000000000ull) return false;
  }
}

// GELU(GN1(h)) of an item's nrows rows into a_s [nrows][MAXH]; hs holds the
// item's h rows (H floats each) already in shared memory.
template <int MAXH>
__device__ __forceinline__ void stage_act(const float* __restrict__ hs, int nrows, int H, float m1, float rs1,
                                          const float* __restrict__ g1w, const float* __restrict__ g1b,
                                          float* __restrict__ a_s) {
  for (int i = threadIdx.x; i < nrows * MAXH; i += blockDim.x) {
    const int r = i / MAXH, j = i - (i / MAXH) * MAXH;
    float v = 0.f;
    if (j < H) v = ub::gelu_erf((hs[r * H + j] - m1) * rs1 * __ldg(g1w + j) + __ldg(g1b + j));
    a_s[i] = v;
  }
}

// Dot product of an activation row (16-byte aligned) with the first HW weights;
// HW is the exact hidden width when it is a multiple of 2 known at compile time.
template <int MAXH, int HW>
__device__ __forceinline__ float dot_a(const float* __restrict__ a, const float (&w)[MAXH]) {
  // Even and odd terms in two packed-FMA partial sums.
  float2 z = make_float2(0.f, 0.f);
#pragma unroll
  for (int j4 = 0; j4 < HW / 4; ++j4) {
    const float4 v = *reinterpret_cast<const float4*>(a + 4 * j4);
    z = ub::fma2(make_float2(v.x, v.y), make_float2(w[4 * j4], w[4 * j4 + 1]), z);
    z = ub::fma2(make_float2(v.z, v.w), make_float2(w[4 * j4 + 2], w[4 * j4 + 3]), z);
  }
  if (HW % 4 == 2) {
    const float2 v = *reinterpret_cast<const float2*>(a + HW - 2);
    z = ub::fma2(v, make_float2(w[HW - 2], w[HW - 1]), z);
  }
  return z.x + z.y;
}


template <int MAXH>
__device__ __forceinline__ void load_w(const float* __restrict__ w2, const float* __restrict__ b2, int H, int cg,
                                       bool live, float (&w)[2 * CPT][MAXH], float (&bz)[2 * CPT]) {
#pragma unroll
  for (int k = 0; k < 2 * CPT; ++k) {
    const int n = 2 * cg * CPT + k;  // z channel (value/gate interleaved)
#pragma unroll
    for (int j = 0; j < MAXH; ++j) w[k][j] = (j < H && live) ? __ldg(w2 + (long long)n * H + j) : 0.f;
    bz[k] = live ? __ldg(b2 + n) : 0.f;
  }
}

static __device__ int g_dconv_error = 0;



// ---------------------------------------------------------------------------
// Register-blocked conv1 for the thin levels (h rows of HP = 4, 8, 12 or 16
// floats, of which the first HW are computed and the rest written as 0).
// A CTA owns C1_IR rows of one group; lane l of warp w computes the HW
// outputs of rows w*32*C1_RT + l + 32*i (i < C1_RT), so one broadcast read of
// the weights of an input (tap, channel) feeds C1_RT*HW FMAs and the
// x reads of a warp hit 32 consecutive rows of a tile with an odd row stride
// (no bank conflicts). Channels are staged C1_CK at a time with their
// dilation halo, zero outside [0, rows).
constexpr int C1_NW = 4;
constexpr int C1_NT = C1_NW * 32;
constexpr int C1_RT = 3;
constexpr int C1_IR = C1_NT * C1_RT;  // rows per CTA
constexpr int C1_CK = 16;              // channels per staged chunk
constexpr int C1_XS = C1_CK + 1;       // staged row stride (floats)
constexpr int C1_MAXDIL = 8;           // largest dilation the launcher accepts
// float4 staging slots per thread: every (row, 4-channel) slot of a chunk with its halo.
constexpr int C1_PF = ((C1_IR + 2 * C1_MAXDIL) * (C1_CK / 4) + C1_NT - 1) / C1_NT;

template <int HP, int HW>
__global__ void __launch_bounds__(C1_NT) dconv_conv1b_kernel(const float* __restrict__ x, long long x_gs, int rows,
                                                             int C, const float* __restrict__ w1,
                                                             const float* __restrict__ b1, int dil,
                                                             float* __restrict__ h, double* __restrict__ stats) {
  extern __shared__ __align__(16) float sm[];
  float* ws = sm;              // [C][3][HP]
  float* xc = sm + 3 * C * HP; // [C1_IR + 2 * dil][C1_XS]
  const int g = blockIdx.y;
  const int r0 = blockIdx.x * C1_IR;
  const float* xg = x + (long long)g * x_gs;
  const int tid = threadIdx.x;
  for (int i = tid; i < HP * 3 * C; i += C1_NT) {
    const int j = i / (3 * C), rem = i - j * 3 * C;
    const int t = rem / C, c = rem - t * C;
    ws[(c * 3 + t) * HP + j] = __ldg(w1 + i);
  }
  const int lr0 = (tid >> 5) * 32 * C1_RT + (tid & 31);
  static_assert(HW % 2 == 0, "pairs of hidden outputs");
  float2 acc[C1_RT][HW / 2];  // (output 2p, output 2p+1) of each row, fed by packed FMAs
#pragma unroll
  for (int p = 0; p < HW / 2; ++p) {
    const float2 b = make_float2(__ldg(b1 + 2 * p), __ldg(b1 + 2 * p + 1));
#pragma unroll
    for (int i = 0; i < C1_RT; ++i) acc[i][p] = b;
  }
  const int last = min(rows, r0 + C1_IR + dil);  // rows past this are never read
  const int nst = min(C1_IR, rows - r0) + 2 * dil;
  // The next chunk's x values are fetched into registers while the current
  // chunk is computed (all C1_PF loads of a thread in flight at once).
  // Slot k of thread tid is staged row rq + PF_ROWS * k, channels [4 q, 4 q + 4) of the chunk.
  constexpr int PF_ROWS = C1_NT / (C1_CK / 4);
  const int q = tid % (C1_CK / 4), rq = tid / (C1_CK / 4);
  const float* xs = xg + (long long)(r0 - dil + rq) * C + 4 * q;  // slot 0 of chunk 0
  float4 pf[C1_PF];
#pragma unroll
  for (int k = 0; k < C1_PF; ++k) {
    const int r = r0 - dil + rq + PF_ROWS * k;
    pf[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (rq + PF_ROWS * k < nst && r >= 0 && r < last)
      pf[k] = __ldg(reinterpret_cast<const float4*>(xs + (long long)PF_ROWS * k * C));
  }
  for (int c0 = 0; c0 < C; c0 += C1_CK) {
    __syncthreads();  // the previous chunk is consumed (and ws is written)
#pragma unroll
    for (int k = 0; k < C1_PF; ++k) {
      if (rq + PF_ROWS * k < nst) {
        float* d = xc + (rq + PF_ROWS * k) * C1_XS + 4 * q;
        d[0] = pf[k].x;
        d[1] = pf[k].y;
        d[2] = pf[k].z;
        d[3] = pf[k].w;
      }
    }
    __syncthreads();
    if (c0 + C1_CK < C) {
      const float* xn = xs + c0 + C1_CK;
#pragma unroll
      for (int k = 0; k < C1_PF; ++k) {
        const int r = r0 - dil + rq + PF_ROWS * k;
        pf[k] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (rq + PF_ROWS * k < nst && r >= 0 && r < last)
          pf[k] = __ldg(reinterpret_cast<const float4*>(xn + (long long)PF_ROWS * k * C));
      }
    }
#pragma unroll 2
    for (int c = 0; c < C1_CK; ++c) {
#pragma unroll
      for (int t = 0; t < 3; ++t) {
        float wv[HP];
#pragma unroll
        for (int j4 = 0; j4 < (HW + 3) / 4; ++j4) {
          const float4 v = *reinterpret_cast<const float4*>(ws + ((c0 + c) * 3 + t) * HP + 4 * j4);
          wv[4 * j4] = v.x;
          wv[4 * j4 + 1] = v.y;
          wv[4 * j4 + 2] = v.z;
          wv[4 * j4 + 3] = v.w;
        }
#pragma unroll
        for (int i = 0; i < C1_RT; ++i) {
          // Staged rows beyond nst are stale but only feed rows >= rows, which are dropped.
          const float xv = xc[(lr0 + 32 * i + t * dil) * C1_XS + c];
          const float2 xx = make_float2(xv, xv);
#pragma unroll
          for (int p = 0; p < HW / 2; ++p) acc[i][p] = ub::fma2(xx, make_float2(wv[2 * p], wv[2 * p + 1]), acc[i][p]);
        }
      }
    }
  }
  float s1 = 0.f, s2 = 0.f;
#pragma unroll
  for (int i = 0; i < C1_RT; ++i) {
    const int r = r0 + lr0 + 32 * i;
    if (r < rows && lr0 + 32 * i < C1_IR) {
      float4* hr = reinterpret_cast<float4*>(h + ((long long)g * rows + r) * HP);
      float hv[HW];
#pragma unroll
      for (int p = 0; p < HW / 2; ++p) {
        hv[2 * p] = acc[i][p].x;
        hv[2 * p + 1] = acc[i][p].y;
      }
#pragma unroll
      for (int j4 = 0; j4 < HP / 4; ++j4) {
        float v[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) v[e] = 4 * j4 + e < HW ? hv[4 * j4 + e] : 0.f;
        hr[j4] = make_float4(v[0], v[1], v[2], v[3]);
      }
#pragma unroll
      for (int j = 0; j < HW; ++j) {
        s1 += hv[j];
        s2 += hv[j] * hv[j];
      }
    }
  }
  const double d1 = ub::warp_sum_d((double)s1), d2 = ub::warp_sum_d((double)s2);
  __shared__ double red[2][C1_NW];
  if ((tid & 31) == 0) {
    red[0][tid >> 5] = d1;
    red[1][tid >> 5] = d2;
  }
  __syncthreads();
  if (tid == 0) {
    double a = 0, b = 0;
    for (int i = 0; i < C1_NW; ++i) {
      a += red[0][i];
      b += red[1][i];
    }
    atomicAdd(stats + 2 * g, a);
    atomicAdd(stats + 2 * g + 1, b);
  }
}

// ---------------------------------------------------------------------------
// Persistent apply for the thin levels: work items of `ir` rows of one group;
// the item's x rows and h rows arrive by bulk copy into a ring of A4_NB
// buffers (loads run A4_AHEAD items ahead), the residual update is computed in
// place in shared memory and leaves by one bulk store per item. A buffer is
// reloaded only after the store issued from it two items earlier has finished
// reading it. Thread (rsub, cg) owns channels [cg*CPT, cg*CPT + CPT) with their
// W2 value/gate rows in registers and walks rows rsub, rsub + RPP, ...
constexpr int A4_NB = 4;
constexpr int A4_AHEAD = 2;

__device__ __forceinline__ void bulk_store(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(sm_u32(src)),
               "r"(bytes)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

template <int MAXH, int HW, bool PRE>
__global__ void __launch_bounds__(NTH2) dconv_apply4_kernel(float* __restrict__ x, long long x_gs,
                                                            const float* __restrict__ h, int groups, int rows, int H,
                                                            int C, const float* __restrict__ st1,
                                                            const float* __restrict__ g1w,
                                                            const float* __restrict__ g1b,
                                                            const float* __restrict__ w2,
                                                            const float* __restrict__ b2,
                                                            const float* __restrict__ st2,
                                                            const float* __restrict__ g2w,
                                                            const float* __restrict__ g2b,
                                                            const float* __restrict__ scale, int ir) {
  extern __shared__ __align__(128) float dsm[];
  const int xt = ir * C, ht = ir * H;    // floats per buffer part (multiples of 4)
  float* a_s = dsm + A4_NB * (xt + ht);  // [ir][MAXH]
  uint64_t* full = reinterpret_cast<uint64_t*>(a_s + ir * MAXH);
  const int CG = C / CPT;
  const int RPP = blockDim.x / CG;
  const int cg = threadIdx.x % CG, rsub = threadIdx.x / CG;
  const bool live = rsub < RPP;
  float w[2 * CPT][MAXH], bz[2 * CPT], gw[2 * CPT], gb[2 * CPT], sc[CPT];
  load_w<MAXH>(w2, b2, H, cg, live, w, bz);
#pragma unroll
  for (int k = 0; k < 2 * CPT; ++k) {
    gw[k] = live ? __ldg(g2w + 2 * cg * CPT + k) : 0.f;
    gb[k] = live ? __ldg(g2b + 2 * cg * CPT + k) : 0.f;
  }
#pragma unroll
  for (int e = 0; e < CPT; ++e) sc[e] = live ? __ldg(scale + cg * CPT + e) : 0.f;
  const int nblk = (rows + ir - 1) / ir;
  const long long items = (long long)groups * nblk;
  if (threadIdx.x == 0) {
    for (int i = 0; i < A4_NB; ++i)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(sm_u32(&full[i])) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  auto item_at = [&](long long it) {
    const int g = (int)(it / nblk);
    const int r0 = (int)(it - (long long)g * nblk) * ir;
    return make_int3(g, r0, min(ir, rows - r0));
  };
  auto issue = [&](long long it, int buf) {
    const int3 t = item_at(it);
    const int g = t.x, r0 = t.y, nr = t.z;
    float* xb = dsm + buf * (xt + ht);
    uint64_t* bar = &full[buf];
    const uint32_t xbytes = (uint32_t)(nr * C * 4), hbytes = (uint32_t)(nr * H * 4);
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sm_u32(bar)), "r"(xbytes + hbytes)
                 : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     sm_u32(xb)),
                 "l"(x + (long long)g * x_gs + (long long)r0 * C), "r"(xbytes), "r"(sm_u32(bar))
                 : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     sm_u32(xb + xt)),
                 "l"(h + ((long long)g * rows + r0) * H), "r"(hbytes), "r"(sm_u32(bar))
                 : "memory");
  };
  if (threadIdx.x == 0)
    for (int i = 0; i < A4_AHEAD && blockIdx.x + (long long)i * gridDim.x < items; ++i)
      issue(blockIdx.x + (long long)i * gridDim.x, i);
  bool ok = true;
  int k = 0;
  for (long long it = blockIdx.x; it < items; it += gridDim.x, ++k) {
    const int b = k % A4_NB;
    const int3 cur = item_at(it);
    const int g = cur.x, r0 = cur.y, nrows = cur.z;
    const long long ahead = it + (long long)A4_AHEAD * gridDim.x;
    if (threadIdx.x == 0 && ahead < items) {
      // Buffer (k + AHEAD) % NB last held item k + AHEAD - NB = k - 2, whose
      // store is the older of the (at most) two committed since.
      asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
      issue(ahead, (k + A4_AHEAD) % A4_NB);
    }
    ok = wait_phase(&full[b], (k / A4_NB) & 1);
    if (__syncthreads_or(!ok)) break;
    float* xs = dsm + b * (xt + ht);
    // PRE: the h rows already hold GELU(GN1(h)) (written by the moments kernel).
    const float* arow = PRE ? xs + xt : a_s;
    const int astride = PRE ? H : MAXH;
    if (!PRE) {
      stage_act<MAXH>(xs + xt, nrows, H, st1[2 * g], st1[2 * g + 1], g1w, g1b, a_s);
      __syncthreads();
    }
    if (live) {
      // GN2 of z = W2 a + b2 folded per item: (z - m2) rstd2 gamma + beta = (W2 a) ga + gc.
      const float m2 = st2[2 * g], rs2 = st2[2 * g + 1];
      float ga[2 * CPT], gc[2 * CPT];
#pragma unroll
      for (int q = 0; q < 2 * CPT; ++q) {
        ga[q] = rs2 * gw[q];
        gc[q] = fmaf(bz[q] - m2, ga[q], gb[q]);
      }
#pragma unroll 2
      for (int r = rsub; r < nrows; r += RPP) {
        const float* a = arow + r * astride;
        float* xr = xs + r * C + cg * CPT;
        float o[CPT];
#pragma unroll
        for (int e = 0; e < CPT; ++e) {
          const float v = fmaf(dot_a<MAXH, HW>(a, w[2 * e]), ga[2 * e], gc[2 * e]);
          const float gt = fmaf(dot_a<MAXH, HW>(a, w[2 * e + 1]), ga[2 * e + 1], gc[2 * e + 1]);
          o[e] = (sc[e] * v) * ub::sigmoid_approx(gt);
        }
        if (CPT == 2) {
          float2 xv = *reinterpret_cast<float2*>(xr);
          xv.x += o[0];
          xv.y += o[CPT - 1];
          *reinterpret_cast<float2*>(xr) = xv;
        } else {
#pragma unroll
          for (int e = 0; e < CPT; ++e) xr[e] += o[e];
        }
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (threadIdx.x == 0)
      bulk_store(x + (long long)g * x_gs + (long long)r0 * C, xs, (uint32_t)(nrows * C * 4));
  }
  if (threadIdx.x == 0) {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    if (!ok) atomicExch(&g_dconv_error, 1);
  }
}

// ---------------------------------------------------------------------------
// GN2 statistics from the moments of the 1x1 conv's input. With a = GELU(GN1(h))
// (HW values per row) and z = W2 a + b2 (2C values per row), the group sums are
//   sum z   = wsum . S1 + n sum(b2)
//   sum z^2 = sum_jk G_jk S2_jk + 2 u . S1 + n sum(b2^2)
// with S1 = sum_r a, S2 = sum_r a a^T, G = W2^T W2, u = W2^T b2, wsum = W2^T 1:
// HW + HW(HW+1)/2 accumulations per row instead of the 2C*HW FMAs of z.
// One warp per item (a group's block of rows), lanes striding its rows; the
// warp's totals go to the group's moments with double atomics.
template <int HW>
__global__ void __launch_bounds__(256) dconv_moments_kernel(const float* h, int groups, int rows,
                                                            int hs, const float* __restrict__ st1,
                                                            const float* __restrict__ g1w,
                                                            const float* __restrict__ g1b,
                                                            double* __restrict__ mom, int rows_per_item,
                                                            float* a_out) {
  constexpr int NP = HW * (HW + 1) / 2;
  constexpr int K = HW + NP;
  const int lane = threadIdx.x & 31;
  const long long nw = (long long)gridDim.x * (blockDim.x >> 5);
  const int nblk = (rows + rows_per_item - 1) / rows_per_item;
  const long long items = (long long)groups * nblk;
  float gw[HW], gb[HW];
#pragma unroll
  for (int j = 0; j < HW; ++j) {
    gw[j] = __ldg(g1w + j);
    gb[j] = __ldg(g1b + j);
  }
  for (long long it = blockIdx.x * (long long)(blockDim.x >> 5) + (threadIdx.x >> 5); it < items; it += nw) {
    const int g = (int)(it / nblk);
    const int r0 = (int)(it - (long long)g * nblk) * rows_per_item;
    const int r1 = min(rows, r0 + rows_per_item);
    const float m1 = __ldg(st1 + 2 * g), rs1 = __ldg(st1 + 2 * g + 1);
    float acc[K];
#pragma unroll
    for (int k = 0; k < K; ++k) acc[k] = 0.f;
    for (int r = r0 + lane; r < r1; r += 32) {
      const float* hr = h + ((long long)g * rows + r) * hs;
      float a[HW];
      // Plain loads: a_out may be h itself (each row is read, then rewritten, by one lane).
#pragma unroll
      for (int j4 = 0; j4 < HW / 4; ++j4) {
        const float4 v = reinterpret_cast<const float4*>(hr)[j4];
        a[4 * j4] = v.x;
        a[4 * j4 + 1] = v.y;
        a[4 * j4 + 2] = v.z;
        a[4 * j4 + 3] = v.w;
      }
      if (HW % 4 == 2) {
        const float2 v = *reinterpret_cast<const float2*>(hr + HW - 2);
        a[HW - 2] = v.x;
        a[HW - 1] = v.y;
      }
#pragma unroll
      for (int j = 0; j < HW; ++j) a[j] = ub::gelu_erf((a[j] - m1) * rs1 * gw[j] + gb[j]);
      if (a_out) {
        // The row of activations for the apply kernel, zero past the computed width.
        float4* ar = reinterpret_cast<float4*>(a_out + ((long long)g * rows + r) * hs);
#pragma unroll
        for (int j4 = 0; j4 < (HW + 3) / 4; ++j4) {
          float v[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) v[e] = 4 * j4 + e < HW ? a[4 * j4 + e] : 0.f;
          ar[j4] = make_float4(v[0], v[1], v[2], v[3]);
        }
        for (int j = 4 * ((HW + 3) / 4); j < hs; ++j) a_out[((long long)g * rows + r) * hs + j] = 0.f;
      }
#pragma unroll
      for (int j = 0; j < HW; ++j) acc[j] += a[j];
      int q = HW;
#pragma unroll
      for (int j = 0; j < HW; ++j)
#pragma unroll
        for (int k = j; k < HW; ++k) {
          acc[q] = fmaf(a[j], a[k], acc[q]);
          ++q;
        }
    }
#pragma unroll
    for (int k = 0; k < K; ++k) acc[k] = ub::warp_sum(acc[k]);
#pragma unroll
    for (int k = 0; k < K; ++k)
      if (lane == (k & 31) && r0 < r1) atomicAdd(mom + (long long)g * K + k, (double)acc[k]);
  }
}

// (sum, sum of squares) of z per group from its moments; coef holds
// [wsum (HW), u (HW), G packed as the upper triangle row by row with the
// off-diagonal entries doubled (NP), sum(b2), sum(b2^2)] in double.
__global__ void dconv_moment_sums_kernel(const double* __restrict__ mom, const double* __restrict__ coef,
                                         int groups, int hw, double n, double* __restrict__ sums) {
  const int K = hw + hw * (hw + 1) / 2;
  for (int g = blockIdx.x * blockDim.x + threadIdx.x; g < groups; g += gridDim.x * blockDim.x) {
    const double* m = mom + (long long)g * K;
    double s = n * coef[2 * hw + K - hw], s2 = n * coef[2 * hw + K - hw + 1];
    for (int j = 0; j < hw; ++j) {
      s += coef[j] * m[j];
      s2 += 2.0 * coef[hw + j] * m[j];
    }
    for (int q = 0; q < K - hw; ++q) s2 += coef[2 * hw + q] * m[hw + q];
    sums[2 * g] = s;
    sums[2 * g + 1] = s2;
  }
}

template <typename K>
unsigned persistent_grid_smem(K kernel, int threads, size_t smem, long long items) {
  int dev = 0, sms = 148, per_sm = 1;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  const long long cap = (long long)sms * per_sm;
  return (unsigned)(items < cap ? items : cap);
}

// Grid of a persistent kernel: every CTA resident at once (items are dealt
// round-robin, so a second wave would double the time of its CTAs' share).
template <typename K>
unsigned persistent_grid(K kernel, size_t smem, long long items) {
  int dev = 0, sms = 148, per_sm = 1;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, NTH2, smem) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  const long long cap = (long long)sms * per_sm;
  return (unsigned)(items < cap ? items : cap);
}

int maxh_for(int H) { return H <= 8 ? 8 : H <= 16 ? 16 : H <= 32 ? 32 : H <= 64 ? 64 : 0; }

}  // namespace

// Hidden rows are padded: h rows, W1 rows, GN1 affine and W2 rows hold
// hs = round_up(hid, 4) values, the ones past hid being zero.
static inline int padded_hidden(int hid) { return (hid + 3) & ~3; }

// Compute width of the fused kernels: the true width when even (their dot
// products take float4/float2 steps), else the padded one (zeros).
static inline int compute_width(int hid) { return hid % 2 == 0 ? hid : padded_hidden(hid); }

extern "C" int unblend_dconv_conv1(const float* x, long long x_gs, int groups, int rows, int c, const float* w1,
                                   const float* b1, int hid, int dil, float* h, double* stats, void* stream) {
  UB_REQUIRE(x && w1 && b1 && h && stats && groups > 0 && rows > 0 && c > 0 && c % 4 == 0);
  UB_REQUIRE(hid > 0 && dil > 0 && dil <= C1_MAXDIL && groups < 65536 && x_gs >= (long long)rows * c);
  const int hs = padded_hidden(hid);
  const int mh = maxh_for(hs);
  UB_REQUIRE(mh > 0);
  cudaStream_t st = ub::as_stream(stream);
  const bool aligned = (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(h) & 15) == 0;
  if (hs <= 16 && c % C1_CK == 0 && x_gs % 4 == 0 && aligned) {
    const size_t smem1 = sizeof(float) * ((size_t)3 * c * hs + (size_t)(C1_IR + 2 * dil) * C1_XS);
    UB_REQUIRE(smem1 <= 200 * 1024);
    dim3 grid1((rows + C1_IR - 1) / C1_IR, groups);
    const int hw = compute_width(hid);
#define UB_C1B(HP, HW)                                                                                          \
  {                                                                                                             \
    cudaFuncSetAttribute(dconv_conv1b_kernel<HP, HW>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem1); \
    dconv_conv1b_kernel<HP, HW><<<grid1, C1_NT, smem1, st>>>(x, x_gs, rows, c, w1, b1, dil, h, stats);          \
  }
    switch (hw) {
      case 2: UB_C1B(4, 2) break;
      case 4: UB_C1B(4, 4) break;
      case 6: UB_C1B(8, 6) break;
      case 8: UB_C1B(8, 8) break;
      case 10: UB_C1B(12, 10) break;
      case 12: UB_C1B(12, 12) break;
      case 14: UB_C1B(16, 14) break;
      case 16: UB_C1B(16, 16) break;
      default: return UNBLEND_ERR_INVALID;
    }
#undef UB_C1B
    UB_CHECK_LAUNCH();
    return 0;
  }
  const size_t smem = sizeof(float) * ((size_t)(ROWS + 2 * dil) * (c + 4) + (size_t)hs * 3 * c);
  UB_REQUIRE(smem <= 220 * 1024);
  dim3 grid((rows + ROWS - 1) / ROWS, groups);
#define UB_LAUNCH(MH)                                                                                         \
  {                                                                                                           \
    cudaFuncSetAttribute(dconv_conv1_kernel<MH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);    \
    dconv_conv1_kernel<MH><<<grid, ROWS, smem, st>>>(x, x_gs, rows, c, w1, b1, hs, dil, h, stats);            \
  }
  if (mh == 8) UB_LAUNCH(8) else if (mh == 16) UB_LAUNCH(16) else if (mh == 32) UB_LAUNCH(32) else UB_LAUNCH(64)
#undef UB_LAUNCH
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_dconv_apply(float* x, long long x_gs, const float* h, int groups, int rows, int hid, int c,
                                   const float* st1, const float* g1w, const float* g1b, const float* w2,
                                   const float* b2, const float* st2, const float* g2w, const float* g2b,
                                   const float* scale, int h_is_act, void* stream) {
  UB_REQUIRE(x && h && w2 && b2 && st2 && g2w && g2b && scale && (h_is_act || (st1 && g1w && g1b)));
  UB_REQUIRE(groups > 0 && rows > 0 && c > 0 && c % 4 == 0 && hid > 0 && groups < 65536);
  UB_REQUIRE(x_gs >= (long long)rows * c && x_gs % 4 == 0);
  const int hs = padded_hidden(hid);
  const int mh = maxh_for(hs);
  UB_REQUIRE(mh > 0);
  cudaStream_t st = ub::as_stream(stream);
  if (mh <= 16 && c % CPT == 0 && c / CPT <= NTH2 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(h) & 15) == 0) {
    const int ir = c <= 48 ? 64 : 32;
    const size_t smem4 = sizeof(float) * ((size_t)A4_NB * ir * (c + hs) + (size_t)ir * mh) + 8 * A4_NB;
    UB_REQUIRE(smem4 <= 200 * 1024);
    const long long items = (long long)groups * ((rows + ir - 1) / ir);
#define UB_AP4K(MH, HW, PRE)                                                                                   \
  {                                                                                                             \
    auto k4 = dconv_apply4_kernel<MH, HW, PRE>;                                                                 \
    cudaFuncSetAttribute(k4, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem4);                          \
    const unsigned g4 = persistent_grid_smem(k4, NTH2, smem4, items);                                           \
    k4<<<g4, NTH2, smem4, st>>>(x, x_gs, h, groups, rows, hs, c, st1, g1w, g1b, w2, b2, st2, g2w, g2b, scale,   \
                                ir);                                                                            \
  }
#define UB_AP4(MH, HW)      \
  if (h_is_act) {           \
    UB_AP4K(MH, HW, true)   \
  } else {                  \
    UB_AP4K(MH, HW, false)  \
  }
    switch (compute_width(hid)) {
      case 2: UB_AP4(8, 2) break;
      case 4: UB_AP4(8, 4) break;
      case 6: UB_AP4(8, 6) break;
      case 8: UB_AP4(8, 8) break;
      case 10: UB_AP4(16, 10) break;
      case 12: UB_AP4(16, 12) break;
      case 14: UB_AP4(16, 14) break;
      case 16: UB_AP4(16, 16) break;
      default: return UNBLEND_ERR_INVALID;
    }
#undef UB_AP4
#undef UB_AP4K
    UB_CHECK_LAUNCH();
    return 0;
  }
  UB_REQUIRE(!h_is_act);  // the general kernel recomputes GELU(GN1(h)) itself
  const size_t smem = sizeof(float) * ((size_t)2 * c * hs + 6 * (size_t)c + c);
  UB_REQUIRE(smem <= 220 * 1024);
  dim3 grid((rows + ROWS - 1) / ROWS, groups);
#define UB_LAUNCH(MH)                                                                                         \
  {                                                                                                           \
    cudaFuncSetAttribute(dconv_apply_kernel<MH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);    \
    dconv_apply_kernel<MH><<<grid, ROWS, smem, st>>>(x, x_gs, h, rows, hs, c, st1, g1w, g1b, w2, b2, st2,     \
                                                     g2w, g2b, scale);                                        \
  }
  if (mh == 8) UB_LAUNCH(8) else if (mh == 16) UB_LAUNCH(16) else if (mh == 32) UB_LAUNCH(32) else UB_LAUNCH(64)
#undef UB_LAUNCH
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_dconv_moments(const float* h, int groups, int rows, int hid, const float* st1,
                                     const float* g1w, const float* g1b, double* moments, float* a_out,
                                     void* stream) {
  UB_REQUIRE(h && st1 && g1w && g1b && moments && groups > 0 && rows > 0 && hid > 0 && hid <= 16);
  UB_REQUIRE((reinterpret_cast<uintptr_t>(h) & 15) == 0 && (reinterpret_cast<uintptr_t>(a_out) & 15) == 0);
  const int hs = padded_hidden(hid);
  const int rpi = 512;  // rows per warp item: 16 per lane
  const long long items = (long long)groups * ((rows + rpi - 1) / rpi);
  const long long warps_needed = items;
  long long blocks = (warps_needed + 7) / 8;
  const long long cap = 148LL * 8;
  if (blocks > cap) blocks = cap;
  cudaStream_t st = ub::as_stream(stream);
#define UB_MOM(HW) dconv_moments_kernel<HW><<<(unsigned)blocks, 256, 0, st>>>(h, groups, rows, hs, st1, g1w, g1b, moments, rpi, a_out)
  switch (compute_width(hid)) {
    case 2: UB_MOM(2); break;
    case 4: UB_MOM(4); break;
    case 6: UB_MOM(6); break;
    case 8: UB_MOM(8); break;
    case 10: UB_MOM(10); break;
    case 12: UB_MOM(12); break;
    case 14: UB_MOM(14); break;
    case 16: UB_MOM(16); break;
    default: return UNBLEND_ERR_INVALID;
  }
#undef UB_MOM
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_dconv_moment_sums(const double* moments, const double* coef, int groups, int rows, int hid,
                                         double* sums, void* stream) {
  UB_REQUIRE(moments && coef && sums && groups > 0 && rows > 0 && hid > 0 && hid <= 16);
  const int hw = compute_width(hid);
  dconv_moment_sums_kernel<<<(groups + 127) / 128, 128, 0, ub::as_stream(stream)>>>(moments, coef, groups, hw,
                                                                                  (double)rows, sums);
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_dconv_error_flag(int* out_host, int clear) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_dconv_error, sizeof(int));
  if (e != cudaSuccess) return (int)e;
  if (out_host) *out_host = v;
  if (clear) {
    int z = 0;
    e = cudaMemcpyToSymbol(g_dconv_error, &z, sizeof(int));
    if (e != cudaSuccess) return (int)e;
  }
  return 0;
}
