// ska_tc.cu -- TMA + tcgen05 token-level SKA kernels (bf16 token tensors).
//
// k_stats_tc: raw per-chunk statistics of one (batch, head, chunk) per CTA
//   G'_c = sum_t z_t z_t^T,  M'_c = sum_t z_{t+1} z_t^T,  C'_c = sum_t v_t z_t^T
// (KLF/koopman_lm/ska.py:96-111: the reference's chunk einsums, the boundary
// transition folded into the chunk that owns z_t) and the chunk's key-norm
// maximum (ska.py:441).  The three products are ONE tensor-core product:
//     [G'; M'; C']  ((2r + P) x r)  =  [Z^T; Z+^T; V^T] (x CS tokens) . Z (CS x r)
// with tokens as K.  TMA writes the three token tiles back to back in the
// canonical no-swizzle layout (ska_tc.cuh), so the stacked A operand is just the
// shared-memory tile read MN-major, and B is its Z part.  bf16 products are exact
// and accumulate in fp32 in TMEM, 128 rows per MMA block.
//
// Every wait is bounded.  A wait that runs out marks the chunk in `status`
// (1: TMA, 2: MMA), waits once more (bounded) for the copies or MMAs in flight,
// poisons the chunk's record with NaN so that it cannot pass silently, frees its
// TMEM and returns.
#include <mutex>

#include <cudaTypedefs.h>

#include "ska_common.cuh"
#include "ska_tc.cuh"

namespace ska {
namespace tc {

constexpr int kStatsThreads = 128;     // 4 warps: TMEM lanes 0-127, one row each
constexpr uint32_t kTmemCols = 512;    // TMEM columns per SM

struct StatsGeom {
  int nb;              // 128-row MMA blocks covering the 2r + P statistic rows
  uint32_t ncols;      // TMEM columns allocated (power of two >= 32)
  uint32_t grp;        // bytes of one feature group: CS tokens x 16 B
  size_t smem;         // dynamic shared memory
};

__host__ __device__ inline StatsGeom stats_geom(int r, int P, int CS) {
  StatsGeom g{};
  g.nb = (2 * r + P + 127) / 128;
  uint32_t need = (uint32_t)(g.nb * r), c = 32;
  while (c < need) c <<= 1;
  g.ncols = c;
  g.grp = (uint32_t)CS * 16u;
  g.smem = (size_t)g.nb * 16 * g.grp + 128;    // + alignment slack
  return g;
}

// s + lo^2 + hi^2 for the two bf16 values packed in w (low half first)
__device__ __forceinline__ float sq2(uint32_t w, float s) {
  const float lo = __uint_as_float(w << 16), hi = __uint_as_float(w & 0xFFFF0000u);
  return fmaf(hi, hi, fmaf(lo, lo, s));
}

__global__ void __launch_bounds__(kStatsThreads, 8) k_stats_tc(const __grid_constant__ CUtensorMap mz,
                                                            const __grid_constant__ CUtensorMap mv, Dims d,
                                                            StatsGeom g, float* __restrict__ stats,
                                                            unsigned long long* __restrict__ cmax,
                                                            int* __restrict__ status) {
  extern __shared__ unsigned char smem_raw[];
  __shared__ uint64_t bar_load, bar_mma;
  __shared__ uint32_t tmem_slot;
  __shared__ unsigned long long red[kStatsThreads / 32];
  unsigned char* tile =
      smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);   // TMA destinations: 128-B aligned
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long q = blockIdx.x;                                  // (b, h, c), c fastest
  const int c = (int)(q % d.C);
  const long long bh = q / d.C;
  const int h = (int)(bh % d.H), b = (int)(bh / d.H);
  const int r = d.r, P = d.P, CS = d.CS, T = d.T;
  const int rows = 2 * r + P;
  unsigned char* tz = tile;                            // Z   : r/8 groups
  unsigned char* tzp = tile + (size_t)(r / 8) * g.grp; // Z+  : r/8 groups (tokens shifted by one)
  unsigned char* tv = tile + (size_t)(r / 4) * g.grp;  // V   : P/8 groups

  if (tid == 0) {
    mbar_init(&bar_load, 1);
    mbar_init(&bar_mma, 1);
    mbar_fence_init();
    tma_prefetch_map(&mz);
    tma_prefetch_map(&mv);
  }
  if (warp == 0) tmem_alloc(&tmem_slot, g.ncols);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tbase = tmem_slot;
  const int t0 = c * CS;

  if (tid == 0) {
    mbar_expect_tx(&bar_load, (uint32_t)rows * (uint32_t)CS * 2u);
    for (int k = 0; k < r / 8; ++k) {
      tma_load_4d(tz + (size_t)k * g.grp, &mz, &bar_load, 8 * k, h, t0, b);
      tma_load_4d(tzp + (size_t)k * g.grp, &mz, &bar_load, 8 * k, h, t0 + 1, b);
    }
    for (int k = 0; k < P / 8; ++k) tma_load_4d(tv + (size_t)k * g.grp, &mv, &bar_load, 8 * k, h, t0, b);
  }
  int st = 0;
  if (!__syncthreads_and(mbar_wait(&bar_load, 0))) {
    st = 1;
    mbar_wait(&bar_load, 0);                           // let copies in flight land
  }

  if (st == 0 && tid == 0) {
    fence_after_sync();
    const uint32_t id = idesc_bf16(128, r, true, true);
    const uint32_t a0 = smem_u32(tile), b0 = smem_u32(tz);
    for (int mb = 0; mb < g.nb; ++mb)
      for (int ks = 0; ks < CS / 16; ++ks)
        mma_bf16(tbase + (uint32_t)(mb * r), sdesc(a0 + (uint32_t)mb * 16u * g.grp + 256u * ks, 128u, g.grp),
                 sdesc(b0 + 256u * ks, 128u, g.grp), id, ks > 0);
    mma_commit(&bar_mma);
  }

  // key-norm maximum over the chunk's real tokens, overlapping the MMAs
  unsigned long long key = 0ull;
  if (st == 0) {
    for (int k = tid; k < CS; k += kStatsThreads) {
      const int t = t0 + k;
      if (t >= T) break;
      float s = 0.f;
      for (int gi = 0; gi < r / 8; ++gi) {
        const uint4 u = *reinterpret_cast<const uint4*>(tz + (size_t)gi * g.grp + (size_t)k * 16);
        s = sq2(u.x, s);
        s = sq2(u.y, s);
        s = sq2(u.z, s);
        s = sq2(u.w, s);
      }
      const unsigned long long kk = pack_max(sqrtf(s), t);
      key = kk > key ? kk : key;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long y = __shfl_xor_sync(0xffffffffu, key, o);
    key = y > key ? y : key;
  }
  if (lane == 0) red[warp] = key;

  if (st == 0 && !__syncthreads_and(mbar_wait(&bar_mma, 0))) {
    st = 2;
    mbar_wait(&bar_mma, 0);                            // let MMAs in flight finish
  }
  __syncthreads();
  fence_after_sync();

  float* rec = stats + q * d.SW;
  if (st == 0) {
    for (int mb = 0; mb < g.nb; ++mb) {
      const int row = mb * 128 + 32 * warp + lane;
      for (int j0 = 0; j0 < r; j0 += 16) {
        float v[16];
        tmem_ld16(tbase + (uint32_t)(mb * r + j0) + ((uint32_t)(32 * warp) << 16), v);
        if (row < rows) {
          float4* dst = reinterpret_cast<float4*>(rec + (size_t)row * r + j0);
#pragma unroll
          for (int e = 0; e < 4; ++e) dst[e] = make_float4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3]);
        }
      }
    }
  } else {
    for (int i = tid; i < rows * r; i += kStatsThreads) rec[i] = __int_as_float(0x7fc00000);
  }
  if (tid == 0) {
    unsigned long long m = red[0];
    for (int w = 1; w < kStatsThreads / 32; ++w) m = red[w] > m ? red[w] : m;
    cmax[q] = m;
    status[q] = st;
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    fence_after_sync();
    tmem_dealloc(tbase, g.ncols);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult qr{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &qr) ==
            cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

static bool stride_ok(long long s_elems, long long extent) {
  return extent == 1 || (s_elems > 0 && (s_elems * 2) % 16 == 0 && s_elems * 2 < (1ll << 40));
}

// A [B, T, H, D] bf16 tensor as a TMA map {D, H, T, B} (the dimension order of
// increasing stride for the usual layouts); box {8, 1, CS, 1}: one feature group
// of CS tokens of one head (16-byte rows), i.e. one column of canonical core
// matrices.  Tokens outside [0, T) read as zeros.
static bool token_map(CUtensorMap* m, const In& x, int B, int T, int H, int D, int CS) {
  PFN_cuTensorMapEncodeTiled_v12000 fn = encode_fn();
  if (!fn) return false;
  const auto sub = [](long long s, long long extent) -> cuuint64_t {
    return (cuuint64_t)(extent == 1 ? 16 : s * 2);   // any valid stride for a unit dimension
  };
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)T, (cuuint64_t)B};
  cuuint64_t strides[3] = {sub(x.sh, H), sub(x.st, T), sub(x.sb, B)};
  cuuint32_t box[4] = {8, 1, (cuuint32_t)CS, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(x.p), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool stats_tc_ok(const Dims& d, const In& z, const In& v) {
  if (d.r % 32 != 0 || d.r > 64 || d.P % 8 != 0 || d.P > 128 || d.CS % 16 != 0 || d.CS > 256) return false;
  const auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!al(z.p) || !al(v.p)) return false;
  return stride_ok(z.st, d.T) && stride_ok(z.sh, d.H) && stride_ok(z.sb, d.B) && stride_ok(v.st, d.T) &&
         stride_ok(v.sh, d.H) && stride_ok(v.sb, d.B);
}

size_t stats_tc_smem(const Dims& d) { return stats_geom(d.r, d.P, d.CS).smem; }

// Resident CTAs per SM are capped so that their TMEM allocations always fit at
// once: when the thread limit allows more CTAs than TMEM does, the shared-memory
// request is raised until one more CTA no longer fits in the SM's 228 KB.
static size_t tmem_safe_smem(uint32_t ncols, int threads, size_t smem) {
  const uint32_t tmem_ctas = kTmemCols / ncols;             // >= 1
  const uint32_t thread_ctas = 2048u / (uint32_t)threads;
  if (tmem_ctas >= thread_ctas) return smem;
  const size_t need = (228u * 1024u) / (tmem_ctas + 1) + 1;
  return smem < need ? need : smem;
}

cudaError_t launch_stats_tc(const Dims& d, const In& z, const In& v, float* stats, unsigned long long* cmax,
                            int* status, cudaStream_t st) {
  CUtensorMap mz, mv;
  if (!token_map(&mz, z, d.B, d.T, d.H, d.r, d.CS) || !token_map(&mv, v, d.B, d.T, d.H, d.P, d.CS))
    return cudaErrorInvalidValue;
  const StatsGeom g = stats_geom(d.r, d.P, d.CS);
  const size_t smem = tmem_safe_smem(g.ncols, kStatsThreads, g.smem);
  cudaError_t e = cudaFuncSetAttribute(k_stats_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const long long n = (long long)d.B * d.H * d.C;
  k_stats_tc<<<(unsigned)n, kStatsThreads, smem, st>>>(mz, mv, d, g, stats, cmax, status);
  return cudaGetLastError();
}

}  // namespace tc
}  // namespace ska
