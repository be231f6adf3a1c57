// ska_step.cu -- recurrent (decode) path of the SKA core: the per-layer state
// after a prompt, and token-by-token steps on it (KLF/koopman_lm/recurrent.py).
//
// State of one (batch, head) series, fp32 (recurrent.py:48-66):
//   G [r][r]  sum_t z_t z_t^T + ridge I        (keys normalised by max_norm)
//   M [r][r]  sum_t z_t z_{t-1}^T
//   C [P][r]  sum_t v_t z_t^T
//   z_last [r], max_norm, flags (bit 0: z_last is set)
// laid out as the arrays of StateLayout below.
//
// k_prefill_state (recurrent.py:129-189) builds it from the forward's saved
// exclusive prefix of the last chunk plus that chunk's own statistics (the prompt
// is not re-read except for its last chunk), scaled by the forward's max key norm.
//
// k_step (recurrent.py:270-375): one warp per series; per token
//   zn = z / max_norm, qn = zq / max_norm (max_norm frozen at its prefill value)
//   G += zn zn^T, M += zn z_last^T (when set), C += v zn^T, z_last = zn
//   L = chol((G + G^T) / 2)  (+1e-4 I where that fails), S = G^-1 = Li^T Li
//   A0 = M S, sigma by 6 power iterations, A = clamp(gamma,1,1.5) / max(sigma,1) A0
//   y = C S L A^K Li qn
// All of it is matrix-vector work: with lane i holding row i of L, row i of M and
// column i of Li, a product X v is a broadcast dot (v_j by shuffle) or a
// butterfly reduce-scatter (sum over lanes of x_lane v_lane), so no r x r product
// is formed; A0 v = M (Li^T (Li v)) and A0^T u = Li^T (Li (M^T u)).
#include <algorithm>

#include "../../include/ska_b200.h"
#include "ska_warp.cuh"

namespace ska {

struct StateLayout {
  size_t G, M, C, zlast, maxnorm, flags, total;
};

StateLayout state_layout(long long B, long long H, long long r, long long P) {
  StateLayout L{};
  const size_t n = (size_t)B * H;
  size_t off = 0;
  L.G = off;       off = align256(off + n * r * r * sizeof(float));
  L.M = off;       off = align256(off + n * r * r * sizeof(float));
  L.C = off;       off = align256(off + n * P * r * sizeof(float));
  L.zlast = off;   off = align256(off + n * r * sizeof(float));
  L.maxnorm = off; off = align256(off + n * sizeof(float));
  L.flags = off;   off = align256(off + n * sizeof(int));
  L.total = off;
  return L;
}

namespace rec {

using namespace wpc;

struct StatePtr {
  float* G;
  float* M;
  float* C;
  float* zlast;
  float* maxnorm;
  int* flags;
};

__device__ __forceinline__ StatePtr state_ptr(char* base, const StateLayout& L) {
  return StatePtr{reinterpret_cast<float*>(base + L.G), reinterpret_cast<float*>(base + L.M),
                  reinterpret_cast<float*>(base + L.C), reinterpret_cast<float*>(base + L.zlast),
                  reinterpret_cast<float*>(base + L.maxnorm), reinterpret_cast<int*>(base + L.flags)};
}

// ---------------------------------------------------------------------------
// fresh state (SKAState.__init__, recurrent.py:52-58): G = ridge I, M = C = 0,
// no z_last, max_norm = 1e-6
// ---------------------------------------------------------------------------
__global__ void k_state_init(Dims d, char* state, StateLayout L) {
  const StatePtr s = state_ptr(state, L);
  const long long n = (long long)d.B * d.H, r = d.r, P = d.P;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n * r * r; i += (long long)gridDim.x * blockDim.x) {
    const long long e = i % (r * r);
    s.G[i] = (e / r == e % r) ? d.ridge : 0.f;
    s.M[i] = 0.f;
  }
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n * P * r; i += (long long)gridDim.x * blockDim.x)
    s.C[i] = 0.f;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n * r; i += (long long)gridDim.x * blockDim.x)
    s.zlast[i] = 0.f;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    s.maxnorm[i] = 1e-6f;
    s.flags[i] = 0;
  }
}

// ---------------------------------------------------------------------------
// prefill state: one CTA per series
// ---------------------------------------------------------------------------
constexpr int kPrefThreads = 128;

template <typename IO>
__global__ void __launch_bounds__(kPrefThreads) k_prefill_state(Dims d, In z, In v, const float* __restrict__ stats,
                                                                const unsigned long long* __restrict__ cmax,
                                                                char* state, StateLayout L) {
  __shared__ unsigned long long red[kPrefThreads / 32];
  const int tid = threadIdx.x;
  const long long bh = blockIdx.x;
  const int h = (int)(bh % d.H), b = (int)(bh / d.H);
  const int r = d.r, P = d.P, C = d.C, T = d.T;
  const StatePtr s = state_ptr(state, L);
  // the series' max key norm, as the forward's consumers take it
  unsigned long long key = 0ull;
  for (int c = tid; c < C; c += kPrefThreads) {
    const unsigned long long x = cmax[bh * C + c];
    key = x > key ? x : key;
  }
  key = warp_max_u64(key);
  if ((tid & 31) == 0) red[tid >> 5] = key;
  __syncthreads();
  key = red[0];
  for (int w = 1; w < kPrefThreads / 32; ++w) key = red[w] > key ? red[w] : key;
  const float m = fmaxf(unpack_norm(key), kNormClamp), im = 1.f / m, im2 = im * im;
  // exclusive prefix of the last chunk + the last chunk's own statistics
  const int cl = C - 1, t0 = cl * d.CS, t1 = T;
  const float* rec = stats + (bh * C + cl) * (long long)d.SW;
  const int n_gm = r * r, n_c = P * r;
  for (int e = tid; e < 2 * n_gm + n_c; e += kPrefThreads) {
    float acc = rec[e];
    if (e < n_gm) {                          // G[i][j] += sum_t z_ti z_tj
      const int i = e / r, j = e % r;
      for (int t = t0; t < t1; ++t) acc = fmaf(ld_tok<IO>(z, b, t, h, i), ld_tok<IO>(z, b, t, h, j), acc);
      s.G[bh * n_gm + e] = acc * im2 + (i == j ? d.ridge : 0.f);
    } else if (e < 2 * n_gm) {               // M[i][j] += sum_t z_{t+1,i} z_tj (t + 1 inside the prompt)
      const int f = e - n_gm, i = f / r, j = f % r;
      for (int t = t0; t + 1 < t1; ++t) acc = fmaf(ld_tok<IO>(z, b, t + 1, h, i), ld_tok<IO>(z, b, t, h, j), acc);
      s.M[bh * n_gm + f] = acc * im2;
    } else {                                 // C[p][j] += sum_t v_tp z_tj
      const int f = e - 2 * n_gm, p = f / r, j = f % r;
      for (int t = t0; t < t1; ++t) acc = fmaf(ld_tok<IO>(v, b, t, h, p), ld_tok<IO>(z, b, t, h, j), acc);
      s.C[bh * n_c + f] = acc * im;
    }
  }
  for (int i = tid; i < r; i += kPrefThreads) s.zlast[bh * r + i] = ld_tok<IO>(z, b, T - 1, h, i) * im;
  if (tid == 0) {
    s.maxnorm[bh] = m;
    s.flags[bh] = 1;
  }
}

// ---------------------------------------------------------------------------
// decode steps: one warp per series, r <= 32
// ---------------------------------------------------------------------------
constexpr int kStepWarps = 4;

// (X v)_lane for X held as COLUMNS (lane k holds X[:, k] in xc): reduce-scatter
__device__ __forceinline__ float mv_cols(const float (&xc)[32], float vk, int lane) {
  float t[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) t[i] = xc[i] * vk;
  return reduce_scatter32(t, lane);
}
// (X v)_lane for X held as ROWS (lane i holds X[i, :] in xr): broadcast dot
__device__ __forceinline__ float mv_rows(const float (&xr)[32], float v) {
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
  for (int j = 0; j < 32; j += 4) {
    s0 = fmaf(xr[j], shfl(v, j), s0);
    s1 = fmaf(xr[j + 1], shfl(v, j + 1), s1);
    s2 = fmaf(xr[j + 2], shfl(v, j + 2), s2);
    s3 = fmaf(xr[j + 3], shfl(v, j + 3), s3);
  }
  return (s0 + s1) + (s2 + s3);
}

template <typename IO>
__global__ void __launch_bounds__(kStepWarps * 32) k_step(Dims d, In z, In zq, In v, const float* __restrict__ gamma_p,
                                                          Out y, char* state, StateLayout L) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const long long bh = (long long)blockIdx.x * kStepWarps + w;
  if (bh >= (long long)d.B * d.H) return;   // warp-uniform; no block barriers below
  const int h = (int)(bh % d.H), b = (int)(bh / d.H);
  const int r = d.r, P = d.P, NPB = p_blocks(P);
  extern __shared__ float4 sm4[];
  float* TG = reinterpret_cast<float*>(sm4) + (size_t)w * (2 + 4) * 1024;   // G, M, then up to 4 C blocks
  float* TM = TG + 1024;
  float* TC = TM + 1024;
  const StatePtr s = state_ptr(state, L);
  float* Gs = s.G + bh * r * r;
  float* Ms = s.M + bh * r * r;
  float* Cs = s.C + bh * (long long)P * r;
  load_mat(TG, Gs, r, r, 1.f, lane);
  load_mat(TM, Ms, r, r, 1.f, lane);
  for (int pb = 0; pb < NPB; ++pb) load_mat(TC + pb * 1024, Cs + pb * 32 * r, P - pb * 32, r, 1.f, lane);
  const float mn = s.maxnorm[bh], imn = 1.f / mn;
  float zl = lane < r ? s.zlast[bh * r + lane] : 0.f;
  bool has_last = (s.flags[bh] & 1) != 0;
  const float gs = fminf(fmaxf(*gamma_p, 1.f), 1.5f);
  __syncwarp();

  for (int t = 0; t < d.T; ++t) {
    // ---- rank-1 updates (recurrent.py:322-334) ----
    const float zn = lane < r ? ld_tok<IO>(z, b, t, h, lane) * imn : 0.f;
    const float qn = lane < r ? ld_tok<IO>(zq, b, t, h, lane) * imn : 0.f;
    float row[32];
    ld_row(row, TG, lane);
#pragma unroll
    for (int j = 0; j < 32; ++j) row[j] = fmaf(zn, shfl(zn, j), row[j]);
    st_row(TG, lane, row);
    float mrow[32];
    ld_row(mrow, TM, lane);
    if (has_last) {
#pragma unroll
      for (int j = 0; j < 32; ++j) mrow[j] = fmaf(zn, shfl(zl, j), mrow[j]);
      st_row(TM, lane, mrow);
    }
    for (int pb = 0; pb < NPB; ++pb) {
      const int p = pb * 32 + lane;
      const float vp = p < P ? ld_tok<IO>(v, b, t, h, p) : 0.f;
      float crow[32];
      ld_row(crow, TC + pb * 1024, lane);
#pragma unroll
      for (int j = 0; j < 32; ++j) crow[j] = fmaf(vp, shfl(zn, j), crow[j]);
      st_row(TC + pb * 1024, lane, crow);
    }
    zl = zn;
    has_last = true;
    __syncwarp();
    // ---- L = chol(sym(G)), jitter where it fails (recurrent.py:341-352) ----
    float gcol[32], g[32], x[32];
    ld_col<32>(gcol, TG, lane);
    bool jit = false;
#pragma unroll 1
    for (int attempt = 0; attempt < 2; ++attempt) {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        float val;
        if (lane < r && j < r) {
          val = 0.5f * (row[j] + gcol[j]);
          if (j == lane && jit) val += kJitter;
        } else {
          val = (j == lane) ? 1.f : 0.f;
        }
        g[j] = val;
      }
      if (chol_inv32(g, x, lane) || jit) break;
      jit = true;
    }
    // g: row lane of L;  x: column lane of Li
    // ---- sigma of A0 = M S (recurrent.py:355, ska.py:41-58) ----
    float vv = lane < r ? rsqrtf((float)r) : 0.f;
    float u = 0.f;
#pragma unroll 1
    for (int it = 0; it <= kPowerIters; ++it) {
      const float a1 = mv_cols(x, vv, lane);           // Li v
      const float a2 = mv_rows(x, a1);                 // Li^T (Li v)   (x as rows of Li^T)
      u = mv_rows(mrow, a2);                           // M S v
      if (it == kPowerIters) break;
      u *= fminf(rsqrtf(warp_sum32(u * u)), 1.f / kPowerEps);
      const float c1 = mv_cols(mrow, u, lane);         // M^T u   (M rows as columns of M^T)
      const float c2 = mv_cols(x, c1, lane);           // Li (M^T u)
      const float c3 = mv_rows(x, c2);                 // Li^T Li M^T u = A0^T u
      vv = c3 * fminf(rsqrtf(warp_sum32(c3 * c3)), 1.f / kPowerEps);
    }
    const float sigma = sqrtf(warp_sum32(u * u));
    const float kk = gs * (1.f / fmaxf(sigma, 1.f));
    // ---- y = C S L A^K Li qn (recurrent.py:357-367) ----
    float wv = mv_cols(x, qn, lane);                   // w_q = Li qn
    for (int k = 0; k < d.K; ++k) {
      const float b1 = mv_cols(x, wv, lane);
      const float b2 = mv_rows(x, b1);
      wv = kk * mv_rows(mrow, b2);                     // A w = kk M S w
    }
    const float zo = mv_rows(g, wv);                   // L w_f
    const float e1 = mv_cols(x, zo, lane);
    const float e2 = mv_rows(x, e1);                   // S L w_f
    for (int pb = 0; pb < NPB; ++pb) {
      float crow[32];
      ld_row(crow, TC + pb * 1024, lane);
      const float yp = mv_rows(crow, e2);              // (C S L w_f)_p
      const int p = pb * 32 + lane;
      if (p < P) st_tok<IO>(y, b, t, h, p, yp);
    }
  }
  // ---- state back to global memory ----
  __syncwarp();
  store_mat(Gs, TG, r, r, 1.f, lane);
  store_mat(Ms, TM, r, r, 1.f, lane);
  for (int pb = 0; pb < NPB; ++pb) store_mat(Cs + pb * 32 * r, TC + pb * 1024, P - pb * 32, r, 1.f, lane);
  if (lane < r) s.zlast[bh * r + lane] = zl;
  if (lane == 0) s.flags[bh] = has_last ? 1 : 0;
}

}  // namespace rec

size_t step_smem(const Dims&) { return (size_t)rec::kStepWarps * 6 * 1024 * sizeof(float); }

cudaError_t launch_state_init(const Dims& d, char* state, const StateLayout& L, cudaStream_t st) {
  const long long n = (long long)d.B * d.H * d.r * d.r;
  const unsigned grid = (unsigned)std::min<long long>((n + 255) / 256 + 1, 4096);
  rec::k_state_init<<<grid, 256, 0, st>>>(d, state, L);
  return cudaGetLastError();
}

template <typename IO>
cudaError_t launch_prefill_state(const Dims& d, const In& z, const In& v, const float* stats,
                                 const unsigned long long* cmax, char* state, const StateLayout& L, cudaStream_t st) {
  rec::k_prefill_state<IO><<<(unsigned)((long long)d.B * d.H), rec::kPrefThreads, 0, st>>>(d, z, v, stats, cmax,
                                                                                         state, L);
  return cudaGetLastError();
}

template <typename IO>
cudaError_t launch_step(const Dims& d, const In& z, const In& zq, const In& v, const float* gamma, const Out& y,
                        char* state, const StateLayout& L, cudaStream_t st) {
  const size_t smem = step_smem(d);
  cudaError_t e = cudaFuncSetAttribute(rec::k_step<IO>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const long long n = (long long)d.B * d.H;
  rec::k_step<IO><<<(unsigned)((n + rec::kStepWarps - 1) / rec::kStepWarps), rec::kStepWarps * 32, smem, st>>>(
      d, z, zq, v, gamma, y, state, L);
  return cudaGetLastError();
}

template cudaError_t launch_prefill_state<float>(const Dims&, const In&, const In&, const float*,
                                                 const unsigned long long*, char*, const StateLayout&, cudaStream_t);
template cudaError_t launch_prefill_state<__nv_bfloat16>(const Dims&, const In&, const In&, const float*,
                                                         const unsigned long long*, char*, const StateLayout&,
                                                         cudaStream_t);
template cudaError_t launch_step<float>(const Dims&, const In&, const In&, const In&, const float*, const Out&, char*,
                                        const StateLayout&, cudaStream_t);
template cudaError_t launch_step<__nv_bfloat16>(const Dims&, const In&, const In&, const In&, const float*,
                                                const Out&, char*, const StateLayout&, cudaStream_t);

}  // namespace ska
