// ska_exact.cu -- fp32 CUDA-core SKA core kernels for sm_100a.
//
// Six kernels, one CTA per (chunk, head, batch) unless noted:
//   forward : k_fwd_stats  raw per-chunk statistics G', M', C' + chunk key-norm max
//             k_scan_fwd   exclusive (decayed) scan over chunks, per (b,h) element
//             k_fwd_chunk  Cholesky (+jitter) / inverse / spectral norm / operator W,
//                          readout y = W qn
//   backward: k_bwd_chunk  recompute the chunk operator, dW and dzq from dy, then the
//                          reverse chain rule down to d(raw statistics), d(max norm)
//                          partial and d(gamma) partial
//             k_scan_bwd   reverse exclusive (decayed) suffix scan; d(max norm) and
//                          d(gamma) reductions
//             k_bwd_tok    per-token dz, dv from the scanned statistic gradients, plus
//                          the arg-max key's share of d(max norm)
//
// Every small matrix lives in shared memory with an odd leading dimension so that
// row- and column-wise accesses are bank-conflict free.  All arithmetic is fp32.
#include <type_traits>

#include "ska_common.cuh"

namespace ska {

// ----------------------------------------------------------------------------
// helpers
// ----------------------------------------------------------------------------

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    unsigned long long y = __shfl_xor_sync(0xffffffffu, x, o);
    x = y > x ? y : x;
  }
  return x;
}

// Block-wide sum; every thread receives the total.  `red` holds >= 32 floats.
__device__ float block_sum(float x, float* red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  x = warp_sum(x);
  __syncthreads();
  if (lane == 0) red[w] = x;
  __syncthreads();
  float s = lane < nw ? red[lane] : 0.f;
  return warp_sum(s);
}

__device__ unsigned long long block_max_u64(unsigned long long x, unsigned long long* red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  x = warp_max_u64(x);
  __syncthreads();
  if (lane == 0) red[w] = x;
  __syncthreads();
  unsigned long long s = lane < nw ? red[lane] : 0ull;
  return warp_max_u64(s);
}

// ---- tensor-core small GEMM (mma.sync m16n8k8 TF32 with a 3-term split) ----
//
// x = hi + lo with hi = tf32(x), lo = tf32(x - hi); a*b ~= hi_a hi_b + hi_a lo_b + lo_a hi_b
// keeps ~fp32 accuracy (error ~2^-21 relative per product) at tensor-core throughput.

__device__ __forceinline__ uint32_t to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ void split_tf32(float x, uint32_t& hi, uint32_t& lo) {
  hi = to_tf32(x);
  lo = to_tf32(x - __uint_as_float(hi));
}
__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// C[M x N] = alpha * op(A) op(B)  (+ C when acc), all operands fp32 in shared memory.
//   op(A)(i,k) = TA ? A[k*lda + i] : A[i*lda + k]
//   op(B)(k,j) = TB ? B[j*ldb + k] : B[k*ldb + j]
// C must not alias A or B.  The calling group is the warp-aligned thread range
// [tid0, tid0 + nthr) given as (tid - tid0, nthr); each warp owns 16x16 output tiles.
// The caller synchronises.
template <bool TA, bool TB>
__device__ void smm(float* __restrict__ Cm, int ldc, const float* __restrict__ A, int lda,
                    const float* __restrict__ Bm, int ldb, int M, int N, int K, float alpha,
                    bool acc, int tid, int nthr) {
  const int lane = tid & 31, warp = tid >> 5, nwarps = nthr >> 5;
  const int g = lane >> 2, t4 = lane & 3;
  const int tm = (M + 15) >> 4, tn = (N + 15) >> 4;
  for (int t = warp; t < tm * tn; t += nwarps) {
    const int i0 = (t / tn) << 4, j0 = (t % tn) << 4;
    const int ra = min(i0 + g, M - 1), rb = min(i0 + g + 8, M - 1);
    const int c0 = min(j0 + g, N - 1), c1 = min(j0 + 8 + g, N - 1);
    float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
    for (int k0 = 0; k0 < K; k0 += 8) {
      const int ka = k0 + t4, kb = k0 + t4 + 4;
      const bool va = ka < K, vb = kb < K;
      const int kas = va ? ka : 0, kbs = vb ? kb : 0;
      float av[4];
      av[0] = TA ? A[kas * lda + ra] : A[ra * lda + kas];
      av[1] = TA ? A[kas * lda + rb] : A[rb * lda + kas];
      av[2] = TA ? A[kbs * lda + ra] : A[ra * lda + kbs];
      av[3] = TA ? A[kbs * lda + rb] : A[rb * lda + kbs];
      if (!va) { av[0] = 0.f; av[1] = 0.f; }
      if (!vb) { av[2] = 0.f; av[3] = 0.f; }
      float bv[4];
      bv[0] = TB ? Bm[c0 * ldb + kas] : Bm[kas * ldb + c0];
      bv[1] = TB ? Bm[c0 * ldb + kbs] : Bm[kbs * ldb + c0];
      bv[2] = TB ? Bm[c1 * ldb + kas] : Bm[kas * ldb + c1];
      bv[3] = TB ? Bm[c1 * ldb + kbs] : Bm[kbs * ldb + c1];
      if (!va) { bv[0] = 0.f; bv[2] = 0.f; }
      if (!vb) { bv[1] = 0.f; bv[3] = 0.f; }
      uint32_t ah[4], al[4], bh[4], bl[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        split_tf32(av[q], ah[q], al[q]);
        split_tf32(bv[q], bh[q], bl[q]);
      }
      mma_tf32(d0, al, bh[0], bh[1]);
      mma_tf32(d0, ah, bl[0], bl[1]);
      mma_tf32(d0, ah, bh[0], bh[1]);
      mma_tf32(d1, al, bh[2], bh[3]);
      mma_tf32(d1, ah, bl[2], bl[3]);
      mma_tf32(d1, ah, bh[2], bh[3]);
    }
    const int r0 = i0 + g, r1 = i0 + g + 8;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float* dd = h ? d1 : d0;
      const int cc = j0 + 8 * h + 2 * t4;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int row = (q < 2) ? r0 : r1, col = cc + (q & 1);
        if (row < M && col < N) {
          float* p = &Cm[row * ldc + col];
          *p = acc ? *p + alpha * dd[q] : alpha * dd[q];
        }
      }
    }
  }
}

// Lower Cholesky in place by ONE warp (left-looking, as LAPACK potf2): lane i
// owns rows i and i+32; column j needs the finished rows < j only, so the warp
// runs without block barriers.  Reads the lower triangle; on success the lower
// triangle holds L and the strict upper triangle is zero.  Returns true
// (uniformly over the warp) at the first non-positive pivot, as potrf's info > 0
// (ska.py:140).  n <= 64.
__device__ bool warp_cholesky(float* G, int n, int ld) {
  const int lane = threadIdx.x & 31;
  for (int j = 0; j < n; ++j) {
    float s[2];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int i = lane + 32 * q;
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
      if (i >= j && i < n) {
        const float* ri = G + i * ld;
        const float* rj = G + j * ld;
        int k = 0;
        for (; k + 4 <= j; k += 4) {
          a0 = fmaf(ri[k], rj[k], a0);
          a1 = fmaf(ri[k + 1], rj[k + 1], a1);
          a2 = fmaf(ri[k + 2], rj[k + 2], a2);
          a3 = fmaf(ri[k + 3], rj[k + 3], a3);
        }
        for (; k < j; ++k) a0 = fmaf(ri[k], rj[k], a0);
        s[q] = ri[j] - ((a0 + a1) + (a2 + a3));
      } else {
        s[q] = 0.f;
      }
    }
    const float dj = __shfl_sync(0xffffffffu, j < 32 ? s[0] : s[1], j & 31);
    if (!(dj > 0.f)) return true;
    const float ljj = sqrtf(dj);
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int i = lane + 32 * q;
      if (i == j) G[i * ld + j] = ljj;
      else if (i > j && i < n) G[i * ld + j] = s[q] / ljj;
    }
    __syncwarp();
  }
  for (int idx = lane; idx < n * n; idx += 32) {
    const int i = idx / n, k = idx % n;
    if (k > i) G[i * ld + k] = 0.f;
  }
  __syncwarp();
  return false;
}

// X = L^{-1} for lower-triangular L, by ONE warp (forward substitution): lane c
// owns columns c and c+32, so every lane reads only its own columns of X.
__device__ void warp_tri_inv(float* X, const float* L, int n, int ld) {
  const int lane = threadIdx.x & 31;
  for (int i = 0; i < n; ++i) {
    const float lii = L[i * ld + i];
    const float* li = L + i * ld;
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int c = lane + 32 * q;
      if (c >= n) continue;
      float v;
      if (c > i) {
        v = 0.f;
      } else if (c == i) {
        v = 1.f / lii;
      } else {
        float a0 = 0.f, a1 = 0.f;
        int k = c;
        for (; k + 2 <= i; k += 2) {
          a0 = fmaf(li[k], X[k * ld + c], a0);
          a1 = fmaf(li[k + 1], X[(k + 1) * ld + c], a1);
        }
        if (k < i) a0 = fmaf(li[k], X[k * ld + c], a0);
        v = -(a0 + a1) / lii;
      }
      X[i * ld + c] = v;
    }
  }
  __syncwarp();
}

// sigma_max estimate of ska.py:41-58 (6 power iterations from v = 1/sqrt(r)),
// computed by one full warp; r <= 64 (two rows per lane).
__device__ float warp_power_sigma(const float* A, int r, int ld) {
  const int lane = threadIdx.x & 31;
  const float v_init = 1.f / sqrtf((float)r);
  float v0 = lane < r ? v_init : 0.f, v1 = lane + 32 < r ? v_init : 0.f;
  float a0 = 0.f, a1 = 0.f;
  for (int it = 0; it <= kPowerIters; ++it) {
    a0 = 0.f;
    a1 = 0.f;
    for (int j = 0; j < r; ++j) {
      const float vj = __shfl_sync(0xffffffffu, j < 32 ? v0 : v1, j & 31);
      if (lane < r) a0 = fmaf(A[lane * ld + j], vj, a0);
      if (lane + 32 < r) a1 = fmaf(A[(lane + 32) * ld + j], vj, a1);
    }
    if (it == kPowerIters) break;  // final A v for sigma
    const float na = fmaxf(sqrtf(warp_sum(a0 * a0 + a1 * a1)), kPowerEps);
    const float u0 = a0 / na, u1 = a1 / na;
    float b0 = 0.f, b1 = 0.f;
    for (int i = 0; i < r; ++i) {
      const float ui = __shfl_sync(0xffffffffu, i < 32 ? u0 : u1, i & 31);
      if (lane < r) b0 = fmaf(A[i * ld + lane], ui, b0);
      if (lane + 32 < r) b1 = fmaf(A[i * ld + lane + 32], ui, b1);
    }
    const float nb = fmaxf(sqrtf(warp_sum(b0 * b0 + b1 * b1)), kPowerEps);
    v0 = b0 / nb;
    v1 = b1 / nb;
  }
  return sqrtf(warp_sum(a0 * a0 + a1 * a1));
}

struct SeriesMax {
  float m;       // clamp(max_t ||z_t||, 1e-6)
  float raw;     // max_t ||z_t||
  int tstar;     // first arg-max token
};

__device__ SeriesMax series_max(const unsigned long long* cmax_bh, int C, unsigned long long* red) {
  unsigned long long k = 0ull;
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    const unsigned long long x = cmax_bh[c];
    k = x > k ? x : k;
  }
  k = block_max_u64(k, red);
  SeriesMax s;
  s.raw = unpack_norm(k);
  s.tstar = unpack_t(k);
  s.m = fmaxf(s.raw, kNormClamp);
  return s;
}

__host__ __device__ __forceinline__ int odd_ld(int n) { return n | 1; }

// ----------------------------------------------------------------------------
// forward: raw chunk statistics
// ----------------------------------------------------------------------------
constexpr int kStatTok = 64;      // tokens staged per tile

template <typename IO>
__global__ void __launch_bounds__(kThreads) k_fwd_stats(Dims d, In z, In v, float* __restrict__ stats,
                                                        unsigned long long* __restrict__ cmax) {
  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int r = d.r, P = d.P, CS = d.CS, T = d.T;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarp = blockDim.x >> 5;
  const int ldz = odd_ld(r), ldv = odd_ld(P);
  extern __shared__ float sm[];
  unsigned long long* red = reinterpret_cast<unsigned long long*>(sm);   // 32 u64
  float* Acc = sm + 64;                    // (2r + P) x ldz : [G ; M ; C]
  float* Zs = Acc + (2 * r + P) * ldz;     // (kStatTok + 1) x ldz
  float* Vs = Zs + (kStatTok + 1) * ldz;   // kStatTok x ldv

  unsigned long long key = 0ull;
  const int tchunk = c * CS;
  for (int k0 = 0; k0 < CS; k0 += kStatTok) {
    const int nk = min(kStatTok, CS - k0);
    __syncthreads();
    // z rows k0 .. k0+nk (one extra: the next token, possibly in the next chunk)
    for (int idx = tid; idx < (nk + 1) * r; idx += blockDim.x) {
      const int k = idx / r, j = idx % r, t = tchunk + k0 + k;
      Zs[k * ldz + j] = (t < T) ? ld_tok<IO>(z, b, t, h, j) : 0.f;
    }
    for (int idx = tid; idx < nk * P; idx += blockDim.x) {
      const int k = idx / P, j = idx % P, t = tchunk + k0 + k;
      Vs[k * ldv + j] = (t < T) ? ld_tok<IO>(v, b, t, h, j) : 0.f;
    }
    __syncthreads();
    for (int k = warp; k < nk; k += nwarp) {   // key-norm maxima over the real tokens
      const int t = tchunk + k0 + k;
      if (t >= T) break;
      float s = 0.f;
      for (int j = lane; j < r; j += 32) s = fmaf(Zs[k * ldz + j], Zs[k * ldz + j], s);
      s = warp_sum(s);
      const unsigned long long kk = pack_max(sqrtf(s), t);
      key = kk > key ? kk : key;
    }
    const bool acc = k0 > 0;
    smm<true, false>(Acc, ldz, Zs, ldz, Zs, ldz, r, r, nk, 1.f, acc, tid, blockDim.x);                  // G += Z^T Z
    smm<true, false>(Acc + r * ldz, ldz, Zs + ldz, ldz, Zs, ldz, r, r, nk, 1.f, acc, tid, blockDim.x);  // M += Z+^T Z
    smm<true, false>(Acc + 2 * r * ldz, ldz, Vs, ldv, Zs, ldz, P, r, nk, 1.f, acc, tid, blockDim.x);    // C += V^T Z
  }
  __syncthreads();
  // record = [G ; M ; C] as a (2r+P) x r row-major matrix
  const size_t bhc = ((size_t)b * d.H + h) * d.C + c;
  float* rec = stats + bhc * d.SW;
  for (int idx = tid; idx < (2 * r + P) * r; idx += blockDim.x) rec[idx] = Acc[(idx / r) * ldz + idx % r];
  key = block_max_u64(key, red);
  if (tid == 0) cmax[bhc] = key;
}

// ----------------------------------------------------------------------------
// exclusive scan over chunks (forward) and exclusive suffix scan (backward)
// ----------------------------------------------------------------------------
// Chunks whose loads go out together before any is added and stored: 16 float4
// per thread (64 registers) keeps every scan CTA of a 96-series problem resident
// while the 32 chunks of a 2048-token series take two L2/DRAM round trips.
constexpr int kScanBatch = 16;

// One thread scans 4 consecutive record floats (a float4 when SW % 4 == 0).
__device__ __forceinline__ void scan_lanes4(float* base, int n4, size_t s, int C, bool reverse, int decay,
                                            float alpha) {
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int c0 = 0; c0 < C; c0 += kScanBatch) {
    float4 x[kScanBatch];
#pragma unroll
    for (int q = 0; q < kScanBatch; ++q) {
      const int c = reverse ? C - 1 - (c0 + q) : c0 + q;
      if (c0 + q < C) {
        if (n4 == 4) {
          x[q] = *reinterpret_cast<const float4*>(base + c * s);
        } else {
          x[q].x = base[c * s];
          x[q].y = n4 > 1 ? base[c * s + 1] : 0.f;
          x[q].z = n4 > 2 ? base[c * s + 2] : 0.f;
          x[q].w = 0.f;
        }
      }
    }
#pragma unroll
    for (int q = 0; q < kScanBatch; ++q) {
      const int c = reverse ? C - 1 - (c0 + q) : c0 + q;
      if (c0 + q < C) {
        if (n4 == 4) {
          *reinterpret_cast<float4*>(base + c * s) = acc;
        } else {
          base[c * s] = acc.x;
          if (n4 > 1) base[c * s + 1] = acc.y;
          if (n4 > 2) base[c * s + 2] = acc.z;
        }
        if (decay) {
          acc.x = fmaf(alpha, acc.x, x[q].x);
          acc.y = fmaf(alpha, acc.y, x[q].y);
          acc.z = fmaf(alpha, acc.z, x[q].z);
          acc.w = fmaf(alpha, acc.w, x[q].w);
        } else {
          acc.x += x[q].x;
          acc.y += x[q].y;
          acc.z += x[q].z;
          acc.w += x[q].w;
        }
      }
    }
  }
}

// Exclusive (decayed) scan of every record float over the chunks of one series.
__global__ void __launch_bounds__(kThreads) k_scan_fwd(Dims d, float* __restrict__ stats) {
  const int e = 4 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (e >= d.SW) return;
  const bool vec = (d.SW & 3) == 0;
  const int n4 = vec ? 4 : min(4, d.SW - e);
  float* base = stats + (size_t)blockIdx.y * d.C * d.SW + e;
  if (vec) {
    scan_lanes4(base, 4, d.SW, d.C, false, d.decay, d.alpha);
  } else {
    for (int q = 0; q < n4; ++q) scan_lanes4(base + q, 1, d.SW, d.C, false, d.decay, d.alpha);
  }
}

// Exclusive (decayed) suffix scan of the statistic gradients, plus the d(max norm)
// and d(gamma) reductions.
__global__ void __launch_bounds__(kThreads) k_scan_bwd(Dims d, float* __restrict__ dstats,
                                                       const float* __restrict__ dmpart,
                                                       const float* __restrict__ dgpart,
                                                       float* __restrict__ dm, float* __restrict__ dgamma) {
  __shared__ float red[32];
  const int e = 4 * (blockIdx.x * blockDim.x + threadIdx.x);
  const int bh = blockIdx.y;
  if (e < d.SW) {
    const bool vec = (d.SW & 3) == 0;
    float* base = dstats + (size_t)bh * d.C * d.SW + e;
    if (vec) {
      scan_lanes4(base, 4, d.SW, d.C, true, d.decay, d.alpha);
    } else {
      const int n4 = min(4, d.SW - e);
      for (int q = 0; q < n4; ++q) scan_lanes4(base + q, 1, d.SW, d.C, true, d.decay, d.alpha);
    }
  }
  if (blockIdx.x == 0) {
    float s = 0.f;
    for (int c = threadIdx.x; c < d.C; c += blockDim.x) s += dmpart[(size_t)bh * d.C + c];
    s = block_sum(s, red);
    if (threadIdx.x == 0) dm[bh] = s;
    if (bh == 0) {
      const size_t n = (size_t)d.B * d.H * d.C;
      float g = 0.f;
      for (size_t i = threadIdx.x; i < n; i += blockDim.x) g += dgpart[i];
      g = block_sum(g, red);
      if (threadIdx.x == 0) *dgamma = g;
    }
  }
}

// ----------------------------------------------------------------------------
// segmented scans: one DRAM round trip per record float
//
// The chunks of one series are cut into G segments of kSegLen consecutive chunks
// (G a power of two <= 16, so C <= 16 * kSegLen).  A CTA takes groups of 32
// consecutive float4 columns of the record, one warp per (group, segment), lane =
// column, so every load and store instruction of a warp covers 512 contiguous bytes.
// Each thread loads all of its segment's chunks at once, scans them locally, and
// the segment totals meet in shared memory:
//   forward (exclusive):  out[c] = sum_{c' < c} a^(c - 1 - c') x[c']
//   backward (suffix):    out[c] = sum_{c' > c} a^(c' - c - 1) x[c']
// (a = decay_alpha for the decay strategy, 1 otherwise): the sums of k_scan_fwd /
// k_scan_bwd in one round trip instead of ceil(C / 16).  Only the last segment
// can be short, and it is never between two others, so the decay between
// segments is a^(kSegLen * gap).
// ----------------------------------------------------------------------------
constexpr int kSegLen = 16;

__host__ __device__ inline int seg_count(int C) {
  int g = 1;
  while (g * kSegLen < C) g <<= 1;
  return g;
}
// G <= 16 (C <= 256): 512 threads at most, so a thread may keep its 16 float4 in registers
bool seg_scan_ok(const Dims& d) { return (d.SW & 3) == 0 && d.C <= 16 * kSegLen; }

__device__ __forceinline__ float4 f4_fma(float a, float4 x, float4 y) {   // a x + y
  return make_float4(fmaf(a, x.x, y.x), fmaf(a, x.y, y.y), fmaf(a, x.z, y.z), fmaf(a, x.w, y.w));
}

// column groups per CTA: 256-thread CTAs for G <= 8 (G = 16: 512 threads)
__host__ __device__ inline int seg_groups(int G) { return G >= 8 ? 1 : 8 / G; }

// the CTA takes seg_groups(G) groups of 32 consecutive columns; thread (x, y):
// column x of group y / G, segment y % G; `tots` holds blockDim.y x 32 float4
template <bool REVERSE>
__device__ __forceinline__ void seg_scan_column(float* series, long long stride, int ncols, int C, float4* tots,
                                                int decay, float alpha) {
  const int G = seg_count(C), seg = threadIdx.y % G, cg = threadIdx.y / G, lane = threadIdx.x;
  const int col = (blockIdx.x * seg_groups(G) + cg) * 32 + lane;
  const bool active = col < ncols;
  const int c0 = seg * kSegLen, n = active ? max(0, min(kSegLen, C - c0)) : 0;
  float* rec0 = series + 4 * (size_t)(active ? col : 0);
  float4 x[kSegLen];
#pragma unroll
  for (int k = 0; k < kSegLen; ++k)
    x[k] = k < n ? *reinterpret_cast<const float4*>(rec0 + (long long)(c0 + k) * stride) : make_float4(0, 0, 0, 0);
  const float a = decay ? alpha : 1.f;
  // local scan in place; tot = the segment's total, weighted toward its far end
  float4 tot = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int i = 0; i < kSegLen; ++i) {
    const int k = REVERSE ? kSegLen - 1 - i : i;
    if (k < n) {
      const float4 xk = x[k];
      x[k] = tot;
      tot = f4_fma(a, tot, xk);
    }
  }
  tots[threadIdx.y * 32 + lane] = tot;
  __syncthreads();
  float aL = 1.f;   // a^kSegLen: the decay across one whole segment
#pragma unroll
  for (int i = 0; i < kSegLen; ++i) aL *= a;
  // offset from the segments before this one (after it, for REVERSE), nearest first
  float4 off = make_float4(0.f, 0.f, 0.f, 0.f);
  float w = 1.f;
  for (int j = 1; j < G; ++j) {
    const int src = REVERSE ? seg + j : seg - j;
    if (src < 0 || src >= G) break;
    off = f4_fma(w, tots[(cg * G + src) * 32 + lane], off);
    w *= aL;
  }
  // out[c] = local[c] + a^(distance to the segment's edge) off
#pragma unroll
  for (int i = 0; i < kSegLen; ++i) {
    const int k = REVERSE ? kSegLen - 1 - i : i;
    if (k < n) {
      float wk = 1.f;
      const int e = REVERSE ? (kSegLen - 1 - k) : k;
      for (int q = 0; q < e; ++q) wk *= a;
      *reinterpret_cast<float4*>(rec0 + (long long)(c0 + k) * stride) = f4_fma(wk, off, x[k]);
    }
  }
}

// grid (ceil(SW / 4 / (32 groups)), B * H), block (32, G * groups)
__global__ void __launch_bounds__(512) k_scan_seg_fwd(Dims d, float* __restrict__ stats) {
  __shared__ float4 tots[32 * 16];
  seg_scan_column<false>(stats + (size_t)blockIdx.y * d.C * d.SW, d.SW, d.SW >> 2, d.C, tots, d.decay, d.alpha);
}

// sum over a (32, blockDim.y) block; every thread receives the total
__device__ float block_sum_2d(float x, float* red) {
  x = warp_sum(x);
  __syncthreads();
  if (threadIdx.x == 0) red[threadIdx.y] = x;
  __syncthreads();
  return warp_sum(threadIdx.x < blockDim.y ? red[threadIdx.x] : 0.f);
}

__global__ void __launch_bounds__(512) k_scan_seg_bwd(Dims d, float* __restrict__ dstats,
                                                       const float* __restrict__ dmpart,
                                                       const float* __restrict__ dgpart,
                                                       float* __restrict__ dm, float* __restrict__ dgamma) {
  __shared__ float4 tots[32 * 16];
  __shared__ float red[32];
  const int bh = blockIdx.y;
  seg_scan_column<true>(dstats + (size_t)bh * d.C * d.SW, d.SW, d.SW >> 2, d.C, tots, d.decay, d.alpha);
  if (blockIdx.x == 0) {   // d(max norm) per series, d(gamma) over everything
    const int tid = threadIdx.y * 32 + threadIdx.x, nt = 32 * blockDim.y;
    float sum = 0.f;
    for (int c = tid; c < d.C; c += nt) sum += dmpart[(size_t)bh * d.C + c];
    sum = block_sum_2d(sum, red);
    if (tid == 0) dm[bh] = sum;
    if (bh == 0) {
      const size_t n = (size_t)d.B * d.H * d.C;
      float g = 0.f;
      for (size_t i = tid; i < n; i += nt) g += dgpart[i];
      g = block_sum_2d(g, red);
      if (tid == 0) *dgamma = g;
    }
  }
}

static dim3 seg_grid(const Dims& d) {
  const int cols_per_cta = 32 * seg_groups(seg_count(d.C));
  return dim3((unsigned)(((d.SW >> 2) + cols_per_cta - 1) / cols_per_cta), d.B * d.H);
}
static dim3 seg_block(const Dims& d) {
  const int G = seg_count(d.C);
  return dim3(32, G * seg_groups(G));
}

// ----------------------------------------------------------------------------
// per-chunk operator (shared by forward and backward)
// ----------------------------------------------------------------------------

// All threads load Gn (+ jitter when `jitter`) into `Lb`; warp 0 factors it and,
// when `Li` is given and the factorisation succeeded, also inverts it.  Returns the
// failure flag (uniform over the block).  Ends with a block barrier.
__device__ bool load_and_factor(const float* rec, int r, int ld, float m2, float ridge, bool jitter,
                                float* Lb, float* Li, int* s_flag) {
  for (int idx = threadIdx.x; idx < r * r; idx += blockDim.x) {
    const int i = idx / r, j = idx % r;
    // ska.py:119,138: G_excl + ridge I, then symmetrise
    float g = 0.5f * (rec[i * r + j] / m2 + rec[j * r + i] / m2);
    if (i == j) g += ridge + (jitter ? kJitter : 0.f);
    Lb[i * ld + j] = g;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const bool f = warp_cholesky(Lb, r, ld);
    if (Li) warp_tri_inv(Li, Lb, r, ld);   // also after a failure, so that the result stays deterministic
    if (threadIdx.x == 0) *s_flag = f ? 1 : 0;
  }
  __syncthreads();
  return *s_flag != 0;
}

// A^K into a buffer chosen among {b_even, b_odd}; returns the pointer holding it
// (may be A itself for K == 1).
__device__ float* matrix_power(float* A, float* b_even, float* b_odd, int r, int ld, int K) {
  if (K == 0) {
    for (int idx = threadIdx.x; idx < r * r; idx += blockDim.x) {
      const int i = idx / r, j = idx % r;
      b_even[i * ld + j] = (i == j) ? 1.f : 0.f;
    }
    __syncthreads();
    return b_even;
  }
  float* cur = A;
  for (int s = 1; s < K; ++s) {
    float* out = (s & 1) ? b_even : b_odd;
    smm<false, false>(out, ld, cur, ld, A, ld, r, r, r, 1.f, false, threadIdx.x, blockDim.x);
    __syncthreads();
    cur = out;
  }
  return cur;
}

// ----------------------------------------------------------------------------
// forward: chunk operator + readout
// ----------------------------------------------------------------------------
constexpr int kReadTok = 64;

template <typename IO>
__global__ void __launch_bounds__(kThreads) k_fwd_chunk(Dims d, In zq, const float* __restrict__ gamma_p, Out y,
                                                        const float* __restrict__ stats,
                                                        const unsigned long long* __restrict__ cmax,
                                                        float* __restrict__ invs_out, int* __restrict__ flags_out) {
  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int r = d.r, P = d.P, CS = d.CS, T = d.T, tid = threadIdx.x, nthr = blockDim.x;
  const int ld = odd_ld(r), MX = max(r, P), bs = MX * ld;
  extern __shared__ float sm[];
  float* red = sm;                                  // 64 floats (32 u64), 256-byte aligned
  float* B0 = sm + 64;
  float* B1 = B0 + bs;
  float* B2 = B1 + bs;
  float* B3 = B2 + bs;
  float* P0 = B3 + bs;
  float* P1 = P0 + bs;
  float* Qs = P1 + bs;                              // kReadTok x ld
  float* Ys = Qs + kReadTok * ld;                   // kReadTok x ldp
  const int ldp = odd_ld(P);
  __shared__ float s_sigma;

  const size_t bh = (size_t)b * d.H + h;
  const size_t bhc = bh * d.C + c;
  const float* rec = stats + bhc * d.SW;
  const SeriesMax sx = series_max(cmax + bh * d.C, d.C, reinterpret_cast<unsigned long long*>(red));
  const float m = sx.m, m2 = m * m;

  // Mn -> B2, Cn -> P0
  for (int idx = tid; idx < r * r; idx += nthr) B2[(idx / r) * ld + idx % r] = rec[r * r + idx] / m2;
  for (int idx = tid; idx < P * r; idx += nthr) P0[(idx / r) * ld + idx % r] = rec[2 * r * r + idx] / m;
  // L -> B0 (jitter retry on failure, ska.py:140-145)
  __shared__ int s_flag;
  int flag = 0;
  if (load_and_factor(rec, r, ld, m2, d.ridge, false, B0, B1, &s_flag)) {
    flag = 1;
    if (load_and_factor(rec, r, ld, m2, d.ridge, true, B0, B1, &s_flag)) flag |= 2;
  }
  smm<true, false>(B0, ld, B1, ld, B1, ld, r, r, r, 1.f, false, tid, nthr);  // S = Li^T Li
  __syncthreads();
  smm<false, false>(B3, ld, B2, ld, B0, ld, r, r, r, 1.f, false, tid, nthr); // A0 = Mn S
  __syncthreads();
  if (tid < 32) {
    const float sg = warp_power_sigma(B3, r, ld);
    if (tid == 0) s_sigma = sg;
  } else {
    smm<false, true>(P1, ld, P0, ld, B1, ld, P, r, r, 1.f, false, tid - 32, nthr - 32);  // X1 = Cn Li^T
  }
  __syncthreads();
  const float invs = 1.f / fmaxf(s_sigma, 1.f);
  const float gs = fminf(fmaxf(*gamma_p, 1.f), 1.5f);
  const float kk = gs * invs;
  for (int idx = tid; idx < r * r; idx += nthr) B3[(idx / r) * ld + idx % r] *= kk;   // A
  __syncthreads();
  float* AK = matrix_power(B3, B0, B2, r, ld, d.K);
  smm<false, false>(P0, ld, P1, ld, AK, ld, P, r, r, 1.f, false, tid, nthr);          // X2 = X1 A^K
  __syncthreads();
  smm<false, false>(P1, ld, P0, ld, B1, ld, P, r, r, 1.f / m, false, tid, nthr);      // W / m
  if (tid == 0) {
    invs_out[bhc] = invs;
    flags_out[bhc] = flag;
  }
  // readout y_t = (W/m) zq_t
  const int tchunk = c * CS;
  for (int k0 = 0; k0 < CS; k0 += kReadTok) {
    const int nk = min(kReadTok, CS - k0);
    __syncthreads();
    for (int idx = tid; idx < nk * r; idx += nthr) {
      const int k = idx / r, j = idx % r, t = tchunk + k0 + k;
      Qs[k * ld + j] = (t < T) ? ld_tok<IO>(zq, b, t, h, j) : 0.f;
    }
    __syncthreads();
    smm<false, true>(Ys, ldp, Qs, ld, P1, ld, nk, P, r, 1.f, false, tid, nthr);   // Y = Qs (W/m)^T
    __syncthreads();
    for (int o = tid; o < nk * P; o += nthr) {
      const int k = o / P, p = o % P, t = tchunk + k0 + k;
      if (t < T) st_tok<IO>(y, b, t, h, p, Ys[k * ldp + p]);
    }
  }
}

// ----------------------------------------------------------------------------
// backward: chunk operator gradients
// ----------------------------------------------------------------------------
constexpr int kBwdTok = 32;

template <typename IO>
__global__ void __launch_bounds__(kThreads) k_bwd_chunk(Dims d, In zq, In dy, const float* __restrict__ gamma_p,
                                                        Out dzq, const float* __restrict__ stats,
                                                        const unsigned long long* __restrict__ cmax,
                                                        const float* __restrict__ invs_in,
                                                        const int* __restrict__ flags_in,
                                                        float* __restrict__ dstats, float* __restrict__ dmpart,
                                                        float* __restrict__ dgpart) {
  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int r = d.r, P = d.P, CS = d.CS, T = d.T, tid = threadIdx.x, nthr = blockDim.x;
  const int ld = odd_ld(r), ldp = odd_ld(P), MX = max(r, P), bs = MX * ld;
  extern __shared__ float sm[];
  float* red = sm;                          // 64 floats (32 u64)
  float* Bf[9];
  for (int i = 0; i < 9; ++i) Bf[i] = sm + 64 + i * bs;
  float* DYs = sm + 64 + 9 * bs;            // kBwdTok x ldp
  float* Qs = DYs + kBwdTok * ldp;          // kBwdTok x ld
  float* DQs = Qs + kBwdTok * ld;           // kBwdTok x ld

  const size_t bh = (size_t)b * d.H + h;
  const size_t bhc = bh * d.C + c;
  const float* rec = stats + bhc * d.SW;
  const SeriesMax sx = series_max(cmax + bh * d.C, d.C, reinterpret_cast<unsigned long long*>(red));
  const float m = sx.m, m2 = m * m, im = 1.f / m;
  const int flag = flags_in[bhc];
  const float invs = invs_in[bhc];
  const float gs = fminf(fmaxf(*gamma_p, 1.f), 1.5f);
  const bool gpass = (*gamma_p >= 1.f) && (*gamma_p <= 1.5f);   // clamp passes grads inclusively
  const float kk = gs * invs;

  // ---- recompute the forward operator (same arithmetic as k_fwd_chunk) ----
  float *bL = Bf[0], *bLi = Bf[1], *bM = Bf[2], *bA = Bf[3];
  float *p0 = Bf[5], *p1 = Bf[6], *p2 = Bf[7], *p3 = Bf[8];
  for (int idx = tid; idx < r * r; idx += nthr) bM[(idx / r) * ld + idx % r] = rec[r * r + idx] / m2;
  for (int idx = tid; idx < P * r; idx += nthr) p0[(idx / r) * ld + idx % r] = rec[2 * r * r + idx] / m;
  __shared__ int s_flag;
  load_and_factor(rec, r, ld, m2, d.ridge, (flag & 1) != 0, bL, bLi, &s_flag);
  smm<true, false>(bL, ld, bLi, ld, bLi, ld, r, r, r, 1.f, false, tid, nthr);  // S (in bL)
  __syncthreads();
  smm<false, false>(bA, ld, bM, ld, bL, ld, r, r, r, 1.f, false, tid, nthr);   // A0
  __syncthreads();
  for (int idx = tid; idx < r * r; idx += nthr) bA[(idx / r) * ld + idx % r] *= kk;  // A
  smm<false, true>(p1, ld, p0, ld, bLi, ld, P, r, r, 1.f, false, tid, nthr);   // X1 = Cn Li^T
  __syncthreads();
  // A^K uses bL (S, dead) / bM (Mn, dead) as ping-pong buffers
  float* AK = matrix_power(bA, bL, bM, r, ld, d.K);
  smm<false, false>(p2, ld, p1, ld, AK, ld, P, r, r, 1.f, false, tid, nthr);   // X2 = X1 A^K
  __syncthreads();
  smm<false, false>(p3, ld, p2, ld, bLi, ld, P, r, r, 1.f, false, tid, nthr);  // W
  __syncthreads();

  // ---- token pass: dW = sum_t dy_t qn_t^T ; dqn_t = W^T dy_t ----
  float* dW = p0;  // Cn is reloaded later
  for (int idx = tid; idx < P * r; idx += nthr) dW[(idx / r) * ld + idx % r] = 0.f;
  float dmq = 0.f;   // <dQn, Qn>
  const int tchunk = c * CS;
  for (int k0 = 0; k0 < CS; k0 += kBwdTok) {
    const int nk = min(kBwdTok, CS - k0);
    __syncthreads();
    for (int idx = tid; idx < nk * P; idx += nthr) {
      const int k = idx / P, p = idx % P, t = tchunk + k0 + k;
      DYs[k * ldp + p] = (t < T) ? ld_tok<IO>(dy, b, t, h, p) : 0.f;
    }
    for (int idx = tid; idx < nk * r; idx += nthr) {
      const int k = idx / r, j = idx % r, t = tchunk + k0 + k;
      Qs[k * ld + j] = (t < T) ? ld_tok<IO>(zq, b, t, h, j) * im : 0.f;
    }
    __syncthreads();
    // dW += DY^T Qn   (P x r, K = nk)
    smm<true, false>(dW, ld, DYs, ldp, Qs, ld, P, r, nk, 1.f, true, tid, nthr);
    // dqn = DY W  (nk x r)
    smm<false, false>(DQs, ld, DYs, ldp, p3, ld, nk, r, P, 1.f, false, tid, nthr);
    __syncthreads();
    for (int o = tid; o < nk * r; o += nthr) {
      const int k = o / r, j = o % r, t = tchunk + k0 + k;
      const float a = DQs[k * ld + j];
      if (t < T) {
        st_tok<IO>(dzq, b, t, h, j, a * im);
        dmq = fmaf(a, Qs[k * ld + j], dmq);
      }
    }
  }
  __syncthreads();

  // ---- reverse chain through W = Cn Li^T A^K Li ----
  // free r-buffers: bL/bM minus AK (and Bf[4])
  float* bFree = (AK == bL) ? bM : bL;
  float* bDLi = bFree;
  float* dX2 = p3;   // W dead
  smm<false, true>(dX2, ld, dW, ld, bLi, ld, P, r, r, 1.f, false, tid, nthr);      // dX2 = dW Li^T
  smm<true, false>(bDLi, ld, p2, ld, dW, ld, r, r, P, 1.f, false, tid, nthr);      // dLi = X2^T dW
  __syncthreads();
  float* dX1 = p0;   // dW dead
  smm<false, true>(dX1, ld, dX2, ld, AK, ld, P, r, r, 1.f, false, tid, nthr);      // dX1 = dX2 AK^T
  __syncthreads();
  float* dAK = (AK == bA || AK == bFree) ? Bf[4] : AK;   // AK dead once dX1 exists
  if (d.K == 0) dAK = Bf[4];
  smm<true, false>(dAK, ld, p1, ld, dX2, ld, r, r, P, 1.f, false, tid, nthr);      // dAK = X1^T dX2
  float* Cn = p2;    // X2 dead: reload Cn
  for (int idx = tid; idx < P * r; idx += nthr) Cn[(idx / r) * ld + idx % r] = rec[2 * r * r + idx] / m;
  __syncthreads();
  float* dCn = p1;   // X1 dead
  smm<false, false>(dCn, ld, dX1, ld, bLi, ld, P, r, r, 1.f, false, tid, nthr);    // dCn = dX1 Li
  smm<true, false>(bDLi, ld, dX1, ld, Cn, ld, r, r, P, 1.f, true, tid, nthr);      // dLi += dX1^T Cn
  __syncthreads();
  float dmc = 0.f;   // <dCn, Cn>
  {
    float* out = dstats + bhc * d.SW + 2 * r * r;
    for (int idx = tid; idx < P * r; idx += nthr) {
      const int p = idx / r, j = idx % r;
      const float g = dCn[p * ld + j];
      dmc = fmaf(g, Cn[p * ld + j], dmc);
      out[idx] = g / m;
    }
  }
  __syncthreads();
  // dA from dAK (A^K): Horner over E_s = dAK (A^T)^s,  H <- E_s + A^T H
  float* dA;
  if (d.K == 0) {
    dA = p0;
    for (int idx = tid; idx < r * r; idx += nthr) dA[(idx / r) * ld + idx % r] = 0.f;
    __syncthreads();
  } else if (d.K == 1) {
    dA = dAK;
  } else {
    float* E = dAK;
    float* H = dAK;
    float* pool[4] = {p0, p1, p2, p3};
    int pi = 0;
    for (int s = 1; s < d.K; ++s) {
      float* En = pool[pi]; pi = (pi + 1) & 3;
      float* Hn = pool[pi]; pi = (pi + 1) & 3;
      smm<false, true>(En, ld, E, ld, bA, ld, r, r, r, 1.f, false, tid, nthr);     // E A^T
      __syncthreads();
      for (int idx = tid; idx < r * r; idx += nthr) Hn[(idx / r) * ld + idx % r] = En[(idx / r) * ld + idx % r];
      __syncthreads();
      smm<true, false>(Hn, ld, bA, ld, H, ld, r, r, r, 1.f, true, tid, nthr);      // += A^T H
      __syncthreads();
      E = En;
      H = Hn;
    }
    dA = H;
  }
  // d gamma partial: A = gs * invs * A0  ->  d gs = <dA, A> / gs
  float dg = 0.f;
  for (int idx = tid; idx < r * r; idx += nthr) {
    const int i = idx / r, j = idx % r;
    dg = fmaf(dA[i * ld + j], bA[i * ld + j], dg);
  }
  // recompute S and reload Mn into free buffers
  float* freeb[4];
  int nf = 0;
  {
    float* cand[7] = {bL, bM, Bf[4], p0, p1, p2, p3};
    for (int i = 0; i < 7 && nf < 4; ++i) {
      float* q = cand[i];
      if (q == dA || q == bDLi || q == bA || q == bLi) continue;
      freeb[nf++] = q;
    }
  }
  float* S = freeb[0];
  float* Mn = freeb[1];
  float* dMn = freeb[2];
  float* dS = freeb[3];
  smm<true, false>(S, ld, bLi, ld, bLi, ld, r, r, r, 1.f, false, tid, nthr);
  for (int idx = tid; idx < r * r; idx += nthr) Mn[(idx / r) * ld + idx % r] = rec[r * r + idx] / m2;
  __syncthreads();
  smm<false, false>(dMn, ld, dA, ld, S, ld, r, r, r, kk, false, tid, nthr);        // dMn = kk dA S
  smm<true, false>(dS, ld, Mn, ld, dA, ld, r, r, r, kk, false, tid, nthr);         // dS = kk Mn^T dA
  __syncthreads();
  float dmm = 0.f;   // <dMn, Mn>
  {
    float* out = dstats + bhc * d.SW + r * r;
    for (int idx = tid; idx < r * r; idx += nthr) {
      const int i = idx / r, j = idx % r;
      const float g = dMn[i * ld + j];
      dmm = fmaf(g, Mn[i * ld + j], dmm);
      out[idx] = g / m2;
    }
  }
  // dS <- dS + dS^T (pairs handled by one thread)
  for (int idx = tid; idx < r * r; idx += nthr) {
    const int i = idx / r, j = idx % r;
    if (j < i) {
      const float s = dS[i * ld + j] + dS[j * ld + i];
      dS[i * ld + j] = s;
      dS[j * ld + i] = s;
    } else if (j == i) {
      dS[i * ld + i] *= 2.f;
    }
  }
  __syncthreads();
  smm<false, false>(bDLi, ld, bLi, ld, dS, ld, r, r, r, 1.f, true, tid, nthr);     // dLi += Li (dS+dS^T)
  __syncthreads();
  // Pm = tril(-tril(dLi) Li^T); only the lower triangle of dLi matters (Li lower)
  float* Pm = dMn;   // written out already
  for (int idx = tid; idx < r * r; idx += nthr) {
    const int i = idx / r, j = idx % r;
    if (j > i) bDLi[i * ld + j] = 0.f;
  }
  __syncthreads();
  smm<false, true>(Pm, ld, bDLi, ld, bLi, ld, r, r, r, -1.f, false, tid, nthr);
  __syncthreads();
  // Pm <- 0.5 (tril(Pm) + tril(Pm,-1)^T): symmetric, diagonal halved
  for (int idx = tid; idx < r * r; idx += nthr) {
    const int i = idx / r, j = idx % r;
    if (j < i) {
      const float s = 0.5f * Pm[i * ld + j];
      Pm[i * ld + j] = s;
      Pm[j * ld + i] = s;
    } else if (j == i) {
      Pm[i * ld + i] *= 0.5f;
    }
  }
  __syncthreads();
  float* T1 = dS;
  smm<false, false>(T1, ld, Pm, ld, bLi, ld, r, r, r, 1.f, false, tid, nthr);      // Pm Li
  __syncthreads();
  float* dGn = S;
  smm<true, false>(dGn, ld, bLi, ld, T1, ld, r, r, r, 1.f, false, tid, nthr);      // Li^T Pm Li
  __syncthreads();
  float dmg = 0.f;   // <dGn, G_excl / m^2>
  {
    float* out = dstats + bhc * d.SW;
    for (int idx = tid; idx < r * r; idx += nthr) {
      const int i = idx / r, j = idx % r;
      const float g = 0.5f * (dGn[i * ld + j] + dGn[j * ld + i]);
      dmg = fmaf(g, 0.5f * (rec[i * r + j] + rec[j * r + i]) / m2, dmg);
      out[idx] = g / m2;
    }
  }
  // d(max norm) partial: -(2<dGn,Gx/m^2> + 2<dMn,Mn> + <dCn,Cn> + <dQn,Qn>) / m
  float tot = 2.f * dmg + 2.f * dmm + dmc + dmq;
  tot = block_sum(tot, red);
  const float dgs = block_sum(dg, red);
  if (tid == 0) {
    dmpart[bhc] = -tot / m;
    dgpart[bhc] = gpass ? dgs / gs : 0.f;
  }
}

// ----------------------------------------------------------------------------
// backward: token pass dz, dv
// ----------------------------------------------------------------------------
constexpr int kTokTile = 64;

template <typename IO>
__global__ void __launch_bounds__(kThreads) k_bwd_tok(Dims d, In z, In v, Out dz, Out dv,
                                                      const float* __restrict__ dstats,
                                                      const unsigned long long* __restrict__ cmax,
                                                      const float* __restrict__ dm) {
  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int r = d.r, P = d.P, CS = d.CS, T = d.T, tid = threadIdx.x, nthr = blockDim.x;
  const int ld = odd_ld(r), ldv = odd_ld(P);
  extern __shared__ float sm[];
  float* G2 = sm;                       // dG + dG^T        r x ld
  float* Ms = G2 + r * ld;              // dM (this chunk)  r x ld
  float* Mp = Ms + r * ld;              // dM (prev chunk)  r x ld
  float* Cs = Mp + r * ld;              // dC               P x ld
  float* Zs = Cs + P * ld;              // (kTokTile + 2) x ld : rows t-1 .. t+nk
  float* Vs = Zs + (kTokTile + 2) * ld; // kTokTile x ldv
  float* DZ = Vs + kTokTile * ldv;      // kTokTile x ld
  float* DV = DZ + kTokTile * ld;       // kTokTile x ldv
  unsigned long long* red = reinterpret_cast<unsigned long long*>(
      (reinterpret_cast<uintptr_t>(DV + kTokTile * ldv) + 7) & ~uintptr_t(7));

  const size_t bh = (size_t)b * d.H + h;
  const size_t bhc = bh * d.C + c;
  const float* rec = dstats + bhc * d.SW;
  for (int idx = tid; idx < r * r; idx += nthr) {
    const int i = idx / r, j = idx % r;
    G2[i * ld + j] = rec[i * r + j] + rec[j * r + i];
    Ms[i * ld + j] = rec[r * r + idx];
    Mp[i * ld + j] = (c > 0) ? rec[r * r + idx - (long long)d.SW] : 0.f;
  }
  for (int idx = tid; idx < P * r; idx += nthr) Cs[(idx / r) * ld + idx % r] = rec[2 * r * r + idx];
  const SeriesMax sx = series_max(cmax + bh * d.C, d.C, red);
  const float dmv = dm[bh];
  const bool route = (sx.raw >= kNormClamp) && (sx.raw > 0.f);

  const int tchunk = c * CS;
  for (int k0 = 0; k0 < CS; k0 += kTokTile) {
    const int nk = min(kTokTile, CS - k0);
    __syncthreads();
    for (int idx = tid; idx < (nk + 2) * r; idx += nthr) {
      const int k = idx / r, j = idx % r, t = tchunk + k0 + k - 1;
      Zs[k * ld + j] = (t >= 0 && t < T) ? ld_tok<IO>(z, b, t, h, j) : 0.f;
    }
    for (int idx = tid; idx < nk * P; idx += nthr) {
      const int k = idx / P, p = idx % P, t = tchunk + k0 + k;
      Vs[k * ldv + p] = (t < T) ? ld_tok<IO>(v, b, t, h, p) : 0.f;
    }
    __syncthreads();
    // dz_t = (dG+dG^T) z_t + dM^T z_{t+1} + dM' z_{t-1} + dC^T v_t   (row form: z_t^T G2 + ...)
    //   dM' is the dM of the chunk owning the transition (t-1 -> t): the previous
    //   chunk for the first token of a chunk (fixed up below).
    const float* Zp = Zs;
    const float* Zc = Zs + ld;
    const float* Zn = Zs + 2 * ld;
    smm<false, false>(DZ, ld, Zc, ld, G2, ld, nk, r, r, 1.f, false, tid, nthr);
    smm<false, false>(DZ, ld, Zn, ld, Ms, ld, nk, r, r, 1.f, true, tid, nthr);
    smm<false, true>(DZ, ld, Zp, ld, Ms, ld, nk, r, r, 1.f, true, tid, nthr);
    smm<false, false>(DZ, ld, Vs, ldv, Cs, ld, nk, r, P, 1.f, true, tid, nthr);
    smm<false, true>(DV, ldv, Zc, ld, Cs, ld, nk, P, r, 1.f, false, tid, nthr);   // dv_t = dC z_t
    __syncthreads();
    if (k0 == 0 && c > 0 && tid < r) {   // first token: (dM_prev - dM) z_{t-1}
      const int i = tid;
      float a = 0.f;
      for (int j = 0; j < r; ++j) a = fmaf(Mp[i * ld + j] - Ms[i * ld + j], Zp[j], a);
      DZ[i] += a;
    }
    __syncthreads();
    for (int o = tid; o < nk * r; o += nthr) {
      const int k = o / r, i = o % r, t = tchunk + k0 + k;
      if (t >= T) continue;
      float a = DZ[k * ld + i];
      if (route && t == sx.tstar) a = fmaf(dmv / sx.raw, Zc[k * ld + i], a);
      st_tok<IO>(dz, b, t, h, i, a);
    }
    for (int o = tid; o < nk * P; o += nthr) {
      const int k = o / P, p = o % P, t = tchunk + k0 + k;
      if (t < T) st_tok<IO>(dv, b, t, h, p, DV[k * ldv + p]);
    }
  }
}

// ----------------------------------------------------------------------------
// host-side launch helpers (called from ska_capi.cu)
// ----------------------------------------------------------------------------

size_t smem_fwd_stats(const Dims& d) {
  const int ldz = odd_ld(d.r), ldv = odd_ld(d.P);
  return ((size_t)64 + (size_t)(2 * d.r + d.P) * ldz + (size_t)(kStatTok + 1) * ldz + (size_t)kStatTok * ldv) *
         sizeof(float);
}
size_t smem_fwd_chunk(const Dims& d) {
  const int ld = odd_ld(d.r), ldp = odd_ld(d.P), MX = d.r > d.P ? d.r : d.P;
  return ((size_t)6 * MX * ld + (size_t)kReadTok * ld + (size_t)kReadTok * ldp + 64) * sizeof(float);
}
size_t smem_bwd_chunk(const Dims& d) {
  const int ld = odd_ld(d.r), ldp = odd_ld(d.P), MX = d.r > d.P ? d.r : d.P;
  return ((size_t)9 * MX * ld + (size_t)kBwdTok * ldp + (size_t)2 * kBwdTok * ld + 64) * sizeof(float);
}
size_t smem_bwd_tok(const Dims& d) {
  const int ld = odd_ld(d.r), ldv = odd_ld(d.P);
  return ((size_t)3 * d.r * ld + (size_t)d.P * ld + (size_t)(kTokTile + 2) * ld + (size_t)kTokTile * ldv +
          (size_t)kTokTile * ld + (size_t)kTokTile * ldv) * sizeof(float) + 8 + 32 * 8;
}

bool warp_path_ok(const Dims& d);
template <typename IO>
cudaError_t launch_fwd_chunk_w(const Dims&, const In&, const float*, const Out&, const float*,
                               const unsigned long long*, float*, int*, float*, unsigned char*, cudaStream_t);
template <typename IO>
cudaError_t launch_bwd_chunk_w(const Dims&, const In&, const In&, const float*, const Out&, const float*,
                               const unsigned long long*, const float*, const int*, float*, float*, float*,
                               cudaStream_t);

namespace tc {
bool stats_tc_ok(const Dims& d, const In& z, const In& v);
bool stats_scan_tc_ok(const Dims& d, const In& z, const In& v);
cudaError_t launch_stats_scan_tc(const Dims& d, const In& z, const In& v, float* stats, unsigned long long* cmax,
                                 int* status, cudaStream_t st);
cudaError_t launch_stats_tc(const Dims& d, const In& z, const In& v, float* stats, unsigned long long* cmax,
                            int* status, cudaStream_t st);
bool tok_bwd_tc_ok(const Dims& d, const In& z, const In& v, const In& dy, const Out& dz, const Out& dv,
                   const Out& dzq, bool dzq_on);
cudaError_t launch_tok_bwd_tc(const Dims& d, const In& z, const In& v, const In& dy, const float* dstats,
                              const unsigned char* wm, const unsigned long long* cmax, const float* dm,
                              const Out& dz, const Out& dv, const Out& dzq, bool dzq_on, int* status,
                              cudaStream_t st);
bool dw_tc_ok(const Dims& d, const In& zq, const In& dy);
cudaError_t launch_dw_tc(const Dims& d, const In& zq, const In& dy, float* dw, int* status, cudaStream_t st);
bool readout_tc_ok(const Dims& d, const In& zq, const Out& y);
bool readout_tc_zq_ok(const Dims& d, const In& zq);
cudaError_t launch_readout_tc(const Dims& d, const In& zq, const unsigned char* wm, const Out& y, bool y32,
                              int* status, cudaStream_t st);
}  // namespace tc
cudaError_t launch_bwd_chunk_s(const Dims& d, const float* gamma, const float* stats, const unsigned long long* cmax,
                               const float* invs, const float* ops, const float* dwraw, float* dstats,
                               float* dmpart, float* dgpart, cudaStream_t st);
bool bwd_ops_tc_ok(const Dims& d);
bool quad_bwd_ok(const Dims& d);
cudaError_t launch_bwd_chunk_q(const Dims& d, const float* gamma, const float* stats, const unsigned long long* cmax,
                               const float* invs, const float* ops, const float* dwraw, float* dstats, float* dmpart,
                               float* dgpart, cudaStream_t st);
cudaError_t launch_bwd_ops_tc(const Dims& d, const float* gamma, const float* stats, const unsigned long long* cmax,
                              const float* invs, const float* ops, const float* dwraw, float* dstats, float* dmpart,
                              float* dgpart, int* status, cudaStream_t st);

bool quad_path_ok(const Dims& d);

// bf16 forwards for 32 < r <= 64 that run the four-warp operator kernel (and keep its
// operators and W / m): the sizes it takes, with a zq the tensor-core readout reads
template <typename IO>
bool quad_fwd(const Dims& d, const In& zq) {
  if constexpr (std::is_same<IO, __nv_bfloat16>::value) {
    return quad_path_ok(d) && tc::readout_tc_zq_ok(d, zq);
  } else {
    return false;
  }
}

// Which backward kernels run (bf16 token tensors with TMA-compatible layouts):
//   full: dW' and dzq on tcgen05, chunk operators without a token pass, from the
//         operators the forward kept (r <= 32, or the four-warp shapes with
//         power_K <= 2)
//   tok : dz, dv on tcgen05; the chunk kernel does the readout's token pass
template <typename IO>
void bwd_tc_paths(const Dims& d, const In& z, const In& zq, const In& v, const In& dy, const Out& dz,
                  const Out& dzq, const Out& dv, bool* full, bool* tok) {
  *full = *tok = false;
  if constexpr (std::is_same<IO, __nv_bfloat16>::value) {
    const bool ops_kept = warp_path_ok(d) || (quad_fwd<IO>(d, zq) && quad_bwd_ok(d));
    *full = ops_kept && tc::dw_tc_ok(d, zq, dy) && tc::tok_bwd_tc_ok(d, z, v, dy, dz, dv, dzq, true);
    *tok = *full || tc::tok_bwd_tc_ok(d, z, v, dy, dz, dv, dzq, false);
  }
}
template void bwd_tc_paths<float>(const Dims&, const In&, const In&, const In&, const In&, const Out&,
                                  const Out&, const Out&, bool*, bool*);
template void bwd_tc_paths<__nv_bfloat16>(const Dims&, const In&, const In&, const In&, const In&, const Out&,
                                          const Out&, const Out&, bool*, bool*);

template <typename K>
static cudaError_t set_smem(K kernel, size_t bytes) {
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

// bf16 token tensors with TMA-compatible alignment take the TMA + tcgen05 statistics kernel
template <typename IO>
bool tc_stats_path(const Dims& d, const In& z, const In& v) {
  if constexpr (std::is_same<IO, __nv_bfloat16>::value) {
    return tc::stats_tc_ok(d, z, v);
  } else {
    return false;
  }
}
template bool tc_stats_path<float>(const Dims&, const In&, const In&);
template bool tc_stats_path<__nv_bfloat16>(const Dims&, const In&, const In&);

bool ops_tc_ok(const Dims& d);
cudaError_t launch_fwd_ops_tc(const Dims& d, const float* gamma, const float* stats, const unsigned long long* cmax,
                              float* invs, int* flags, float* lit, float* ops, unsigned char* wm, int* status,
                              cudaStream_t st);
cudaError_t launch_fwd_chunk_q(const Dims& d, const float* gamma, const float* stats, const unsigned long long* cmax,
                               float* invs, int* flags, float* lis, float* ops, unsigned char* wm, cudaStream_t st);

// bf16 tensors on the warp or four-warp path whose zq and y the tensor-core readout
// can take
template <typename IO>
bool fwd_tc_readout(const Dims& d, const In& zq, const Out& y) {
  if constexpr (std::is_same<IO, __nv_bfloat16>::value) {
    return (warp_path_ok(d) || quad_path_ok(d)) && tc::readout_tc_ok(d, zq, y);
  } else {
    return false;
  }
}
template bool fwd_tc_readout<float>(const Dims&, const In&, const Out&);
template bool fwd_tc_readout<__nv_bfloat16>(const Dims&, const In&, const Out&);

// y32: bf16 inputs with an fp32 y (the tensor-core readout path only; the caller checks
// fwd_tc_readout first).  keep_ops: write the chunk operators the backward reads
// (the saved buffer has room for them).
template <typename IO>
cudaError_t launch_fwd(const Dims& d, const In& z, const In& zq, const In& v, const float* gamma, const Out& y,
                       const SavedLayout& L, char* saved, cudaStream_t st, bool y32, bool keep_ops) {
  float* stats = reinterpret_cast<float*>(saved + L.stats);
  unsigned long long* cmax = reinterpret_cast<unsigned long long*>(saved + L.cmax);
  float* invs = reinterpret_cast<float*>(saved + L.invs);
  int* flags = reinterpret_cast<int*>(saved + L.flags);
  const dim3 grid(d.C, d.H, d.B);
  cudaError_t e;
  const size_t s1 = smem_fwd_stats(d), s3 = smem_fwd_chunk(d);
  if ((e = set_smem(k_fwd_stats<IO>, s1)) != cudaSuccess) return e;
  if ((e = set_smem(k_fwd_chunk<IO>, s3)) != cudaSuccess) return e;
  prof_record(0, st);
  bool fused = false;   // statistics and scan in one kernel
  if (tc_stats_path<IO>(d, z, v)) {
    int* status = reinterpret_cast<int*>(saved + L.status);
    fused = tc::stats_scan_tc_ok(d, z, v);
    e = fused ? tc::launch_stats_scan_tc(d, z, v, stats, cmax, status, st)
              : tc::launch_stats_tc(d, z, v, stats, cmax, status, st);
    if (e != cudaSuccess) return e;
  } else {
    // no tensor-core kernel writes the status entries: they read as "no wait expired"
    const size_t n = (size_t)d.B * d.H * d.C * sizeof(int);
    if ((e = cudaMemsetAsync(saved + L.status, 0, n, st)) != cudaSuccess) return e;
    k_fwd_stats<IO><<<grid, kThreads, s1, st>>>(d, z, v, stats, cmax);
  }
  prof_record(1, st);
  if (!fused) {
    if (seg_scan_ok(d))
      k_scan_seg_fwd<<<seg_grid(d), seg_block(d), 0, st>>>(d, stats);
    else
      k_scan_fwd<<<dim3((d.SW + 4 * kThreads - 1) / (4 * kThreads), d.B * d.H), kThreads, 0, st>>>(d, stats);
  }
  prof_record(2, st);
  bool tc_read = false;   // readout as its own tensor-core kernel
  if (warp_path_ok(d)) {
    // bf16 forwards write W / m for the tensor-core readout and backward, and keep
    // the chunk operators for the backward when the buffer has room for them
    const bool keep = std::is_same<IO, __nv_bfloat16>::value;
    float* ops = keep && keep_ops ? reinterpret_cast<float*>(saved + L.ops) : nullptr;
    unsigned char* wm = keep ? reinterpret_cast<unsigned char*>(saved + L.wm) : nullptr;
    tc_read = fwd_tc_readout<IO>(d, zq, y);
    if (keep && tc_read && ops_tc_ok(d)) {   // four chunks per CTA on tcgen05
      e = launch_fwd_ops_tc(d, gamma, stats, cmax, invs, flags, reinterpret_cast<float*>(saved + L.lis), ops, wm,
                            reinterpret_cast<int*>(saved + L.status),
                            st);
    } else {
      const Out ychunk = tc_read ? Out{nullptr, 0, 0, 0} : y;
      e = launch_fwd_chunk_w<IO>(d, zq, gamma, ychunk, stats, cmax, invs, flags, ops, wm, st);
    }
    if (e != cudaSuccess) return e;
  } else if (quad_fwd<IO>(d, zq)) {   // 32 < r <= 64: four-warp operators, tensor-core readout
    float* ops = keep_ops ? reinterpret_cast<float*>(saved + L.ops) : nullptr;
    if ((e = launch_fwd_chunk_q(d, gamma, stats, cmax, invs, flags, reinterpret_cast<float*>(saved + L.lis), ops,
                                reinterpret_cast<unsigned char*>(saved + L.wm), st)) != cudaSuccess)
      return e;
    tc_read = fwd_tc_readout<IO>(d, zq, y);
    // a y the tensor-core readout cannot store: the one-CTA kernel writes it (and
    // the same invs and flags)
    if (!tc_read) k_fwd_chunk<IO><<<grid, kThreads, s3, st>>>(d, zq, gamma, y, stats, cmax, invs, flags);
  } else {
    k_fwd_chunk<IO><<<grid, kThreads, s3, st>>>(d, zq, gamma, y, stats, cmax, invs, flags);
  }
  prof_record(3, st);
  if (tc_read) {
    const unsigned char* wm = reinterpret_cast<const unsigned char*>(saved + L.wm);
    if ((e = tc::launch_readout_tc(d, zq, wm, y, y32, reinterpret_cast<int*>(saved + L.status), st)) != cudaSuccess)
      return e;
  }
  prof_record(9, st);
  return cudaGetLastError();
}

template <typename IO>
cudaError_t launch_bwd(const Dims& d, const In& z, const In& zq, const In& v, const float* gamma, const In& dy,
                       const SavedLayout& L, const char* saved, const ScratchLayout& S, char* scratch,
                       const Out& dz, const Out& dzq, const Out& dv, float* dgamma, cudaStream_t st) {
  const float* stats = reinterpret_cast<const float*>(saved + L.stats);
  const unsigned long long* cmax = reinterpret_cast<const unsigned long long*>(saved + L.cmax);
  const float* invs = reinterpret_cast<const float*>(saved + L.invs);
  const int* flags = reinterpret_cast<const int*>(saved + L.flags);
  float* dstats = reinterpret_cast<float*>(scratch + S.dstats);
  float* dmpart = reinterpret_cast<float*>(scratch + S.dmpart);
  float* dgpart = reinterpret_cast<float*>(scratch + S.dgpart);
  float* dm = reinterpret_cast<float*>(scratch + S.dm);
  const dim3 grid(d.C, d.H, d.B);
  cudaError_t e;
  const size_t s1 = smem_bwd_chunk(d), s3 = smem_bwd_tok(d);
  if ((e = set_smem(k_bwd_chunk<IO>, s1)) != cudaSuccess) return e;
  if ((e = set_smem(k_bwd_tok<IO>, s3)) != cudaSuccess) return e;
  bool full = false, tc_tok = false;
  bwd_tc_paths<IO>(d, z, zq, v, dy, dz, dzq, dv, &full, &tc_tok);
  float* dw = reinterpret_cast<float*>(scratch + S.dw);
  // the bf16 forward on the warp path (which the full tensor-core backward implies)
  // kept the chunk operators and W / m
  const float* ops = reinterpret_cast<const float*>(saved + L.ops);
  const unsigned char* wm = reinterpret_cast<const unsigned char*>(saved + L.wm);
  int* status = reinterpret_cast<int*>(scratch + S.status);
  prof_record(4, st);
  // the readout-gradient kernel writes every chunk's status; otherwise start from 0
  // (the token kernel ORs its own code into bits 2-3)
  if (!full && (e = cudaMemsetAsync(status, 0, (size_t)d.B * d.H * d.C * sizeof(int), st)) != cudaSuccess)
    return e;
  if (full && (e = tc::launch_dw_tc(d, zq, dy, dw, status, st)) != cudaSuccess) return e;
  prof_record(5, st);
  if (full) {
    // r <= 32: four chunks per CTA on tcgen05 (r % 16 == 0, power_K <= 2), else warp
    // per chunk; 32 < r <= 64: four warps per chunk
    if (!warp_path_ok(d))
      e = launch_bwd_chunk_q(d, gamma, stats, cmax, invs, ops, dw, dstats, dmpart, dgpart, st);
    else if (bwd_ops_tc_ok(d))
      e = launch_bwd_ops_tc(d, gamma, stats, cmax, invs, ops, dw, dstats, dmpart, dgpart, status, st);
    else
      e = launch_bwd_chunk_s(d, gamma, stats, cmax, invs, ops, dw, dstats, dmpart, dgpart, st);
    if (e != cudaSuccess) return e;
  } else if (warp_path_ok(d)) {
    if ((e = launch_bwd_chunk_w<IO>(d, zq, dy, gamma, dzq, stats, cmax, invs, flags, dstats, dmpart, dgpart,
                                    st)) != cudaSuccess)
      return e;
  } else {
    k_bwd_chunk<IO><<<grid, kThreads, s1, st>>>(d, zq, dy, gamma, dzq, stats, cmax, invs, flags, dstats, dmpart,
                                               dgpart);
  }
  prof_record(6, st);
  if (seg_scan_ok(d))
    k_scan_seg_bwd<<<seg_grid(d), seg_block(d), 0, st>>>(d, dstats, dmpart, dgpart, dm, dgamma);
  else
    k_scan_bwd<<<dim3((d.SW + 4 * kThreads - 1) / (4 * kThreads), d.B * d.H), kThreads, 0, st>>>(d, dstats, dmpart, dgpart,
                                                                                     dm, dgamma);
  prof_record(7, st);
  if (tc_tok) {
    if ((e = tc::launch_tok_bwd_tc(d, z, v, dy, dstats, wm, cmax, dm, dz, dv, dzq, full, status, st)) !=
        cudaSuccess)
      return e;
  } else {
    k_bwd_tok<IO><<<grid, kThreads, s3, st>>>(d, z, v, dz, dv, dstats, cmax, dm);
  }
  prof_record(8, st);
  return cudaGetLastError();
}

template cudaError_t launch_fwd<float>(const Dims&, const In&, const In&, const In&, const float*, const Out&,
                                       const SavedLayout&, char*, cudaStream_t, bool, bool);
template cudaError_t launch_fwd<__nv_bfloat16>(const Dims&, const In&, const In&, const In&, const float*,
                                               const Out&, const SavedLayout&, char*, cudaStream_t, bool, bool);
template cudaError_t launch_bwd<float>(const Dims&, const In&, const In&, const In&, const float*, const In&,
                                       const SavedLayout&, const char*, const ScratchLayout&, char*, const Out&,
                                       const Out&, const Out&, float*, cudaStream_t);
template cudaError_t launch_bwd<__nv_bfloat16>(const Dims&, const In&, const In&, const In&, const float*,
                                               const In&, const SavedLayout&, const char*, const ScratchLayout&,
                                               char*, const Out&, const Out&, const Out&, float*, cudaStream_t);

}  // namespace ska
