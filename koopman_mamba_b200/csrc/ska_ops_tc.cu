// ska_ops_tc.cu -- forward chunk operators of rank r <= 32 on tcgen05, four
// chunks per CTA (bf16 token tensors).
//
// The per-chunk algebra of the forward (ska.py:136-176): Cholesky factor of
// Gn and its inverse Li, S = Li^T Li, A0 = Mn S, the power iteration for
// sigma(A0) (ska.py:41-58), A = clamp(gamma) / max(sigma, 1) A0, A^K,
// U = A^K Li, V = Li^T U and W / m = (C / m) V / m, for four chunks at a time.
// Warp w of a CTA owns chunk 4 * blockIdx.x + w.  Its lanes hold one matrix row
// each in registers, as in the warp kernels, and run the Cholesky, the inverse and
// the power iteration on shuffles -- all four warps at once.  The r x r products
// of the four chunks go to the tensor core together: their left operands are
// stacked into one 128-row operand and their right operands side by side into
// one 128-column operand, so that one M = 128, N = 128 product holds each chunk's
// product as a diagonal 32 x 32 block (the off-diagonal blocks are computed and
// never read).  Warp w reads its block from TMEM lanes 32w..32w+31, columns
// 32w..32w+31: exactly the rows its lanes own.
//
// Operands are fp32 values split into bf16 hi + lo planes and a product is the
// three terms hi*hi + hi*lo + lo*hi (kind::f16, fp32 accumulation), about 2^-16
// relative -- the precision of the other tensor-core products of the bf16 path.
//
// Shared-memory operand slots (SWIZZLE_NONE canonical form).  A slot holds the
// four chunks' 32 x 32 tiles as a hi plane and then a lo plane of 8 KB each, in
// 8 x 8 core matrices of 128 contiguous bytes (8 rows of 16 bytes, each 8
// consecutive columns of one row).  A lane holding row i of a matrix Y of chunk j
// writes it in one of two arrangements:
//   R (rows stacked):    core matrix (i / 8, cg) at (4 j + i / 8) * 512 + cg * 128;
//                        the left operand Y (K-major) or the right operand Y^T
//                        (K-major);
//   C (columns stacked): core matrix (i / 8, cg) at (4 j + cg) * 512 + (i / 8) * 128;
//                        the left operand Y^T (MN-major) or the right operand Y
//                        (MN-major).
// In both, core matrices adjacent in K are 128 bytes apart (LBO) and adjacent in
// M or N 512 bytes apart (SBO); a 16-wide K step advances 256 bytes.
//
// W = Cn V has P rows per chunk: the P-row blocks of (4 / NPB) chunks stack into
// one 128-row left operand (slot 1 + g for group g), and group g's product
// (N = 128 / NPB: the V tiles of its chunks) lands in TMEM columns
// [g * 128 / NPB, (g + 1) * 128 / NPB).
#include "ska_tc.cuh"
#include "ska_warp.cuh"

namespace ska {
namespace otc {

using wpc::ChunkId;

constexpr int kOpsThreads = 128;           // 4 warps, one chunk each
constexpr uint32_t kPlane = 8192;          // one bf16 plane: 4 chunks x 32 x 32 x 2 bytes
constexpr uint32_t kSlot = 2 * kPlane;     // hi plane, then lo plane
constexpr uint32_t kOpsCols = 128;         // TMEM columns per CTA (4 CTAs per SM fill the 512)

__host__ __device__ constexpr int ops_npb(int P) { return P <= 32 ? 1 : (P <= 64 ? 2 : 4); }
__host__ __device__ constexpr int ops_slots(int npb) { return npb <= 2 ? 3 : 1 + npb; }

// 16-byte unit (row, column group cg): R arrangement, row 0..127 of the stacked rows
__device__ __forceinline__ uint32_t unit_r(int row, int cg) {
  return (uint32_t)(row >> 3) * 512u + (uint32_t)cg * 128u + (uint32_t)(row & 7) * 16u;
}
// C arrangement, row i (0..31) of chunk j's tile
__device__ __forceinline__ uint32_t unit_c(int j, int i, int cg) {
  return (uint32_t)(4 * j + cg) * 512u + (uint32_t)(i >> 3) * 128u + (uint32_t)(i & 7) * 16u;
}

// this lane's fp32 row v -> bf16 hi and lo units of a slot
template <bool COLS>
__device__ __forceinline__ void put_row(unsigned char* slot, int j, int i, const float (&v)[32]) {
#pragma unroll
  for (int cg = 0; cg < 4; ++cg) {
    float x[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) x[e] = v[8 * cg + e];
    uint4 hi, lo;
    split_bf16x8(x, hi, lo);
    const uint32_t o = COLS ? unit_c(j, i, cg) : unit_r(32 * j + i, cg);
    *reinterpret_cast<uint4*>(slot + o) = hi;
    *reinterpret_cast<uint4*>(slot + kPlane + o) = lo;
  }
}
// both arrangements of one row (one split)
__device__ __forceinline__ void put_row_rc(unsigned char* slot_r, unsigned char* slot_c, int j, int i,
                                           const float (&v)[32]) {
#pragma unroll
  for (int cg = 0; cg < 4; ++cg) {
    float x[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) x[e] = v[8 * cg + e];
    uint4 hi, lo;
    split_bf16x8(x, hi, lo);
    const uint32_t orr = unit_r(32 * j + i, cg), oc = unit_c(j, i, cg);
    *reinterpret_cast<uint4*>(slot_r + orr) = hi;
    *reinterpret_cast<uint4*>(slot_r + kPlane + orr) = lo;
    *reinterpret_cast<uint4*>(slot_c + oc) = hi;
    *reinterpret_cast<uint4*>(slot_c + kPlane + oc) = lo;
  }
}
// R arrangement at stacked row `row` (the P-row blocks of the W operand)
__device__ __forceinline__ void put_row_at(unsigned char* slot, int row, const float (&v)[32]) {
#pragma unroll
  for (int cg = 0; cg < 4; ++cg) {
    float x[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) x[e] = v[8 * cg + e];
    uint4 hi, lo;
    split_bf16x8(x, hi, lo);
    *reinterpret_cast<uint4*>(slot + unit_r(row, cg)) = hi;
    *reinterpret_cast<uint4*>(slot + kPlane + unit_r(row, cg)) = lo;
  }
}

// D[tmem_d, N columns] (=|+=) op(A) op(B): two 16-wide K steps x three split terms.
// a, b: shared addresses of the operands' hi planes; *_mn: C arrangement (MN-major).
__device__ __forceinline__ void mma3(uint32_t tmem_d, uint32_t a, bool a_mn, uint32_t b, bool b_mn, int N,
                                     bool acc) {
  const uint32_t id = tc::idesc_bf16(128, N, a_mn, b_mn);
#pragma unroll
  for (int ks = 0; ks < 2; ++ks) {
    const uint64_t ah = tc::sdesc(a + 256u * ks, 128u, 512u), al = tc::sdesc(a + kPlane + 256u * ks, 128u, 512u);
    const uint64_t bh = tc::sdesc(b + 256u * ks, 128u, 512u), bl = tc::sdesc(b + kPlane + 256u * ks, 128u, 512u);
    tc::mma_bf16(tmem_d, ah, bh, id, acc || ks > 0);
    tc::mma_bf16(tmem_d, ah, bl, id, true);
    tc::mma_bf16(tmem_d, al, bh, id, true);
  }
}

// this thread's operand writes -> visible to the tensor core; then the whole CTA
__device__ __forceinline__ void operands_ready() {
  tc::fence_async_smem();
  tc::fence_before_sync();
  __syncthreads();
}

// wait for the product committed to `bar`; a first wait that gives up (limit)
// still drains the product with the full limit (it owns TMEM and the slots)
__device__ __forceinline__ bool product_wait(uint64_t* bar, uint32_t& phase, uint32_t limit) {
  bool ok = tc::mbar_wait(bar, phase, limit);
  if (!ok) tc::mbar_wait(bar, phase, tc::kWaitLimit);
  phase ^= 1u;
  tc::fence_after_sync();
  return ok;
}

// row `lane` of a kept operator (32 x 32 fp32, element (i, j) at
// ((j / 4) * 32 + i) * 4 + j % 4): one coalesced 512-byte store per column quad
__device__ __forceinline__ void store_op(float* dst, const float (&v)[32], int lane) {
  float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
  for (int k = 0; k < 8; ++k) d4[k * 32 + lane] = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
}

// The backward's record rows (lane = row, 128-byte rows: each warp store
// instruction would touch 32 lines) go out as one bulk copy per block from a 4 KB
// staging buffer per warp, off the load/store path the operand loads use (the
// backward kernel 115.4 -> 112.7 us at B=8, H=12, L=2048, r=32, P=64; the
// forward's kept operators are already stored 512 contiguous bytes per
// instruction and stay plain stores).
// Lane 0 issues every bulk copy of its warp and, before the buffer is rewritten,
// waits until the previous one has read it.  Call with the whole warp.
constexpr uint32_t kStageBytes = 4096;

__device__ __forceinline__ void stage_acquire(int lane) {
  if (lane == 0) tc::bulk_wait_read();
  __syncwarp();
}
__device__ __forceinline__ void stage_release(void* gdst, const float* stg, uint32_t bytes, int lane) {
  tc::fence_async_smem();   // the staged values, to the bulk copy's proxy
  __syncwarp();
  if (lane == 0) {
    tc::bulk_store(gdst, tc::smem_u32(stg), bytes);
    tc::bulk_commit();
  }
}

// column `col` of the n x n row-major matrix src (zero past n); for a fixed k
// the warp reads one contiguous row
__device__ __forceinline__ void ld_gmem_col(float (&v)[32], const float* src, int col, int n) {
  const bool cv = col < n;
  float x[32];
#pragma unroll
  for (int k = 0; k < 32; ++k) x[k] = __ldg(src + (size_t)(k < n ? k : 0) * n + (cv ? col : 0));
#pragma unroll
  for (int k = 0; k < 32; ++k) v[k] = (cv && k < n) ? x[k] : 0.f;
}

// Gn = sym(G) / m^2 + ridge I (+ jitter), factored with its inverse (ska.py:136-145):
// x = row `lane` of Li^T (column `lane` of L^{-1}); cb: 32 floats of the warp's shared
// memory for the column broadcasts.  Returns the jitter flags.  R16: r <= 16, the
// factorisation stops after 16 steps (the rest is identity padding).
template <bool R16 = false>
__device__ __forceinline__ int factor_invert_rows(const Dims& d, const float* rec, int lane, float im2,
                                                  float (&x)[32], float* cb) {
  const int r = d.r;
  int flag = 0;
  bool jit = false;
#pragma unroll 1
  for (int attempt = 0; attempt < 2; ++attempt) {
    float g[32];
    {
      float grow[32], gcol[32];
      wpc::ld_gmem_row(grow, rec, lane, r, r, 1.f);
      ld_gmem_col(gcol, rec, lane, r);
      wpc::build_gram_row(g, grow, gcol, lane, r, im2, d.ridge, jit ? kJitter : 0.f);
    }
    if (jit) flag |= 1;
    if (wpc::chol_inv32_bc<R16>(g, x, cb, lane, 16)) break;
    if (jit) {
      flag |= 2;
      break;
    }
    jit = true;
  }
  return flag;
}

// row p of chunk q's W / m -> the bf16 hi and lo planes of the readout operand
// ([2][r/8][P][8]); NaN when the chunk's products failed
__device__ __forceinline__ void store_wm_row(unsigned char* wq, const float (&u)[32], int p, int P, int r,
                                             bool nan) {
#pragma unroll
  for (int ng = 0; ng < 4; ++ng) {
    if (8 * ng >= r) break;
    float x[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) x[e] = nan ? __int_as_float(0x7fc00000) : u[8 * ng + e];
    uint4 hi, lo;
    split_bf16x8(x, hi, lo);
    *reinterpret_cast<uint4*>(wq + (size_t)ng * P * 16 + (size_t)p * 16) = hi;
    *reinterpret_cast<uint4*>(wq + (size_t)P * r * 2 + (size_t)ng * P * 16 + (size_t)p * 16) = lo;
  }
}

// L2 prefetch of [p, p + bytes) by one bulk-copy-engine request (p 16-byte
// aligned, bytes a multiple of 16), issued by lane 0
__device__ __forceinline__ void prefetch_l2(const void* p, int bytes, int lane) {
  if (lane == 0) asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// The values stay untouched until here: a computation that consumes a load may
// not be scheduled before this point (the product waits sit between a load and
// its use, so that the load's latency overlaps the product).
__device__ __forceinline__ void touch(float4& x) {
  asm volatile("" : "+f"(x.x), "+f"(x.y), "+f"(x.z), "+f"(x.w));
}
__device__ __forceinline__ void touch32(float (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 32; j += 4) asm volatile("" : "+f"(v[j]), "+f"(v[j + 1]), "+f"(v[j + 2]), "+f"(v[j + 3]));
}

// A row of an r-column (r = 16 or 32) row-major fp32 matrix, issued now and
// finished later (scaled, zero when the row is past the matrix)
struct RowLd {
  float4 x[8];
};
__device__ __forceinline__ void row_issue(RowLd& L, const float* src, int row, int nrows, int r) {
  const float4* p = reinterpret_cast<const float4*>(src + (size_t)(row < nrows ? row : 0) * r);
#pragma unroll
  for (int k = 0; k < 8; ++k) L.x[k] = (4 * k < r) ? __ldg(p + k) : make_float4(0.f, 0.f, 0.f, 0.f);
}
__device__ __forceinline__ void row_finish(float (&v)[32], RowLd& L, bool rv, float scale) {
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    touch(L.x[k]);
    v[4 * k] = rv ? L.x[k].x * scale : 0.f;
    v[4 * k + 1] = rv ? L.x[k].y * scale : 0.f;
    v[4 * k + 2] = rv ? L.x[k].z * scale : 0.f;
    v[4 * k + 3] = rv ? L.x[k].w * scale : 0.f;
  }
}

// row `lane` of a kept operator (layout of store_op), loaded raw
__device__ __forceinline__ void ld_op_row(float (&v)[32], const float* src, int lane) {
  const float4* s4 = reinterpret_cast<const float4*>(src);
  float4 x[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) x[k] = __ldg(s4 + k * 32 + lane);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    v[4 * k] = x[k].x;
    v[4 * k + 1] = x[k].y;
    v[4 * k + 2] = x[k].z;
    v[4 * k + 3] = x[k].w;
  }
}

// the same, issued now and finished later
__device__ __forceinline__ void row_issue_op(RowLd& L, const float* src, int lane) {
  const float4* s4 = reinterpret_cast<const float4*>(src);
#pragma unroll
  for (int k = 0; k < 8; ++k) L.x[k] = __ldg(s4 + k * 32 + lane);
}
__device__ __forceinline__ void row_finish_op(float (&v)[32], RowLd& L) {
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    touch(L.x[k]);
    v[4 * k] = L.x[k].x;
    v[4 * k + 1] = L.x[k].y;
    v[4 * k + 2] = L.x[k].z;
    v[4 * k + 3] = L.x[k].w;
  }
}

// Columns of a 32 x 32 matrix whose row `lane` the lanes hold, through a warp's
// own fp32 tile in shared memory: rows 0-15 at lo16, rows 16-31 at hi16 (two
// 2 KB pieces), 16-byte chunks XOR-swizzled by row so that the row writes and
// the column reads are both conflict-free.
__device__ __forceinline__ float* tile_row(unsigned char* lo16, unsigned char* hi16, int i) {
  return reinterpret_cast<float*>((i < 16 ? lo16 : hi16) + (i & 15) * 128);
}
__device__ __forceinline__ void rows_to_cols(float (&col)[32], const float (&row)[32], unsigned char* lo16,
                                             unsigned char* hi16, int lane) {
  float4* w4 = reinterpret_cast<float4*>(tile_row(lo16, hi16, lane));
#pragma unroll
  for (int q = 0; q < 8; ++q) w4[q ^ (lane & 7)] = make_float4(row[4 * q], row[4 * q + 1], row[4 * q + 2], row[4 * q + 3]);
  __syncwarp();
#pragma unroll
  for (int i = 0; i < 32; ++i) col[i] = tile_row(lo16, hi16, i)[(((lane >> 2) ^ (i & 7)) << 2) | (lane & 3)];
  __syncwarp();
}

// sigma_max estimate of ska.py:41-58 (6 power iterations from v = 1/sqrt(r);
// x / max(||x||, 1e-8) taken as x * min(rsqrt(||x||^2), 1e8)) for the matrix
// whose row `lane` is a and column `lane` is ac: each iterate is broadcast
// through 32 floats of the warp's shared memory (vb) and the products are row
// dots, so that an iteration costs two broadcasts and two warp sums.
__device__ __forceinline__ float power_sigma_bc(const float (&a)[32], const float (&ac)[32], float* vb, int lane,
                                                int r) {
  float v = lane < r ? rsqrtf((float)r) : 0.f;
  float u = 0.f;
  const float4* vb4 = reinterpret_cast<const float4*>(vb);
#pragma unroll 1
  for (int it = 0; it <= kPowerIters; ++it) {
    vb[lane] = v;
    __syncwarp();
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 x = vb4[q];
      s0 = fmaf(a[4 * q], x.x, s0);
      s1 = fmaf(a[4 * q + 1], x.y, s1);
      s2 = fmaf(a[4 * q + 2], x.z, s2);
      s3 = fmaf(a[4 * q + 3], x.w, s3);
    }
    u = (s0 + s1) + (s2 + s3);                         // (A v)_lane
    __syncwarp();
    if (it == kPowerIters) break;
    u *= fminf(rsqrtf(wpc::warp_sum32(u * u)), 1.f / kPowerEps);
    vb[lane] = u;
    __syncwarp();
    s0 = s1 = s2 = s3 = 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 x = vb4[q];
      s0 = fmaf(ac[4 * q], x.x, s0);
      s1 = fmaf(ac[4 * q + 1], x.y, s1);
      s2 = fmaf(ac[4 * q + 2], x.z, s2);
      s3 = fmaf(ac[4 * q + 3], x.w, s3);
    }
    const float wv = (s0 + s1) + (s2 + s3);            // (A^T u)_lane
    __syncwarp();
    v = wv * fminf(rsqrtf(wpc::warp_sum32(wv * wv)), 1.f / kPowerEps);
  }
  return sqrtf(wpc::warp_sum32(u * u));
}

// CTAs of a persistent operator kernel: as many per SM as its TMEM share
// (per_sm), its registers and its shared memory allow, never more than the groups.
// The register and shared-memory limits are worked out here from the kernel's
// attributes (228 KB of shared memory per SM, 1 KB of it reserved per CTA; 64 K
// registers, allocated per warp in units of 256).
static cudaError_t persistent_grid(const void* fn, size_t smem, int per_sm, long long groups, unsigned* grid) {
  int dev = 0, sms = 0;
  cudaError_t e;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
  // all of the unified L1 / shared storage as shared memory
  if ((e = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, 100)) != cudaSuccess) return e;
  cudaFuncAttributes fa{};
  if ((e = cudaFuncGetAttributes(&fa, fn)) != cudaSuccess) return e;
  const int warp_regs = ((fa.numRegs * 32 + 255) / 256) * 256;
  const int by_regs = 65536 / (warp_regs * (kOpsThreads / 32));
  const int by_smem = (int)((228u * 1024u) / (smem + fa.sharedSizeBytes + 1024u));
  int occ = per_sm;
  occ = by_regs < occ ? by_regs : occ;
  occ = by_smem < occ ? by_smem : occ;
  if (occ < 1) occ = 1;
  const long long n = (long long)sms * occ;
  *grid = (unsigned)(groups < n ? groups : n);
  return cudaSuccess;
}

// ---------------------------------------------------------------------------
// k_factor32: the Cholesky + inverse of every chunk's Gram matrix (r <= 32), one
// warp per chunk, ahead of the operator kernel: there each warp factored its own
// chunk in registers (~11K cycles of a group) before the group's first product.
// Here the factorisations of many chunks run at once with next to no shared
// memory.  Writes Li^T in the kept-operator layout (store_op) and the jitter
// flags (ska.py:140-145).  R16: r <= 16, 16 steps.
// ---------------------------------------------------------------------------
constexpr int kFac32Warps = 4;

template <bool R16>
__global__ void __launch_bounds__(kFac32Warps * 32, 3) k_factor32(Dims d, const float* __restrict__ stats,
                                                              const unsigned long long* __restrict__ cmax,
                                                              float* __restrict__ lit, int* __restrict__ flags_out) {
  __shared__ __align__(16) float cb[kFac32Warps][32];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long q = (long long)blockIdx.x * kFac32Warps + w;
  if (q >= (long long)d.B * d.H * d.C) return;   // warp-uniform; no block barriers
  const ChunkId id = wpc::chunk_id(d, q);
  const float m = wpc::series_norm(cmax, id, d.C, lane), im = 1.f / m;
  float x[32];
  const int flag = factor_invert_rows<R16>(d, stats + q * d.SW, lane, im * im, x, cb[w]);
  if (lane == 0) flags_out[q] = flag;
  store_op(lit + q * (long long)kOpFloats, x, lane);
}

// ---------------------------------------------------------------------------
// forward.  Persistent: CTA b takes the chunk groups b, b + gridDim.x, ... and
// starts the next group's record on its way to L2 when it begins a group.  The
// chunks' Li^T rows come from k_factor32, except in the r <= 16 instance (R16),
// which factors its chunks itself (16 steps; a separate kernel cost more there
// than it saved: at B=256, H=4, L=1024, r=16, P=32 the forward went 0.332 -> 0.342
// ms, against 0.337 -> 0.328 ms fwd+bwd at B=8, H=12, L=2048, r=32, P=64).
// ---------------------------------------------------------------------------
template <int NPB, bool R16 = false>
__global__ void __launch_bounds__(kOpsThreads, 3) k_fwd_ops_tc(Dims d, const float* __restrict__ gamma_p,
                                                               const float* __restrict__ stats,
                                                               const unsigned long long* __restrict__ cmax,
                                                               float* __restrict__ invs_out,
                                                               int* __restrict__ flags_out,
                                                               const float* __restrict__ lit,
                                                               float* __restrict__ ops_out,
                                                               unsigned char* __restrict__ wm_out,
                                                               int* __restrict__ status) {
  constexpr int kCpg = 4 / NPB;            // chunks per W group
  constexpr int kGroupCols = 128 / NPB;    // TMEM columns (N) of a W group
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_slot;
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  const long long nq = (long long)d.B * d.H * d.C;
  const long long ngroups = (nq + 3) / 4;
  const int r = d.r, P = d.P;
  {
    const long long q = (long long)blockIdx.x * 4 + w < nq ? (long long)blockIdx.x * 4 + w : nq - 1;
    prefetch_l2(stats + q * d.SW, d.SW * 4, lane);
  }
  unsigned char* S0 = smem;
  unsigned char* S1 = smem + kSlot;
  unsigned char* S2 = smem + 2 * kSlot;
  const uint32_t a0 = tc::smem_u32(S0), a1 = a0 + kSlot, a2 = a0 + 2 * kSlot;

  if (w == 0) tc::tmem_alloc(&tmem_slot, kOpsCols);
  if (tid == 0) {
    tc::mbar_init(&bar, 1);
    tc::mbar_fence_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_slot;
  const uint32_t tmine = tmem + ((uint32_t)(32 * w) << 16) + (uint32_t)(32 * w);   // this warp's diagonal block
  const float gs = fminf(fmaxf(*gamma_p, 1.f), 1.5f);
  uint32_t phase = 0;

#pragma unroll 1
  for (long long gi = blockIdx.x; gi < ngroups; gi += gridDim.x) {
    const long long q0 = gi * 4;
    const bool valid = q0 + w < nq;
    const long long q = valid ? q0 + w : nq - 1;   // a spare warp redoes the last chunk and stores nothing
    RowLd ll;                                          // Li^T rows (k_factor32)
    if (!R16) row_issue_op(ll, lit + q * (long long)kOpFloats, lane);
    if (gi + gridDim.x < ngroups) {
      long long qn = (gi + gridDim.x) * 4 + w;
      qn = qn < nq ? qn : nq - 1;
      prefetch_l2(stats + qn * d.SW, d.SW * 4, lane);
      if (!R16) prefetch_l2(lit + qn * (long long)kOpFloats, kOpFloats * 4, lane);
    }
    bool ok = true;
    const ChunkId id = wpc::chunk_id(d, q);
    const float* rec = stats + q * d.SW;
    // operators are kept only when the caller gave the whole saved buffer
    float* opq = ops_out ? ops_out + q * (long long)(kNumOps * kOpFloats) : nullptr;
    const bool keep = valid && opq;
    const float m = wpc::series_norm(cmax, id, d.C, lane), im = 1.f / m, im2 = im * im;
    float t[32];

    // Li^T rows -> R(Li^T) in S0: the left operand Li^T and the right operand Li
    {
      float x[32];
      if (R16) {
        // S2's part of this warp (free until C(S) is written) holds the column broadcasts
        const int flag = factor_invert_rows<true>(d, rec, lane, im2, x, reinterpret_cast<float*>(S2 + 2048 * w));
        if (valid && lane == 0) flags_out[q] = flag;
      } else {
        row_finish_op(x, ll);
      }
      if (keep) store_op(opq + kOpLi * kOpFloats, x, lane);
      put_row<false>(S0, w, lane, x);
    }
    operands_ready();
    if (tid == 0) {
      tc::fence_after_sync();
      mma3(tmem, a0, false, a0, false, 128, false);     // S = Li^T Li
      tc::mma_commit(&bar);
    }
    {
      RowLd ml;
      row_issue(ml, rec + r * r, lane, r, r);           // M rows, while S is formed
      ok &= product_wait(&bar, phase, d.wlim);
      float mn[32];
      row_finish(mn, ml, lane < r, im2);
      put_row<false>(S1, w, lane, mn);                  // R(Mn)
    }
    tc::tmem_ld32(tmine, t);
    if (keep) store_op(opq + kOpS * kOpFloats, t, lane);
    put_row<true>(S2, w, lane, t);                      // C(S): the right operand S
    operands_ready();
    if (tid == 0) {
      tc::fence_after_sync();
      mma3(tmem, a1, false, a2, true, 128, false);      // A0 = Mn S
      tc::mma_commit(&bar);
    }
    ok &= product_wait(&bar, phase, d.wlim);
    tc::tmem_ld32(tmine, t);
    float invs;
    {
      // S1 and S2 are free: this warp's part of each holds its column tile and the
      // broadcast vector (each warp touches only its own rows of a slot)
      float ac[32];
      rows_to_cols(ac, t, S1 + 2048 * w, S1 + kPlane + 2048 * w, lane);
      const float sigma = power_sigma_bc(t, ac, reinterpret_cast<float*>(S2 + 2048 * w), lane, r);   // ska.py:41-58
      invs = 1.f / fmaxf(sigma, 1.f);
    }
    const float kk = gs * invs;                         // ska.py:167-169
#pragma unroll
    for (int j = 0; j < 32; ++j) t[j] *= kk;
    if (keep) store_op(opq + kOpA * kOpFloats, t, lane);
    put_row_rc(S1, S2, w, lane, t);                     // R(A): left operand; C(A): right operand
    if (d.K == 0) {
#pragma unroll
      for (int j = 0; j < 32; ++j) t[j] = (j == lane) ? 1.f : 0.f;
      put_row<false>(S1, w, lane, t);
    }
#pragma unroll 1
    for (int s = 1; s < d.K; ++s) {                     // A^(s+1) = A^s A
      operands_ready();
      if (tid == 0) {
        tc::fence_after_sync();
        mma3(tmem, a1, false, a2, true, 128, false);
        tc::mma_commit(&bar);
      }
      ok &= product_wait(&bar, phase, d.wlim);
      tc::tmem_ld32(tmine, t);
      put_row<false>(S1, w, lane, t);
    }
    if (keep) store_op(opq + kOpAK * kOpFloats, t, lane);
    operands_ready();
    if (tid == 0) {
      tc::fence_after_sync();
      mma3(tmem, a1, false, a0, false, 128, false);     // U = A^K Li
      tc::mma_commit(&bar);
    }
    ok &= product_wait(&bar, phase, d.wlim);
    tc::tmem_ld32(tmine, t);
    if (keep) store_op(opq + kOpU * kOpFloats, t, lane);
    put_row<true>(S2, w, lane, t);                      // C(U)
    operands_ready();
    if (tid == 0) {
      tc::fence_after_sync();
      mma3(tmem, a0, false, a2, true, 128, false);      // V = Li^T U
      tc::mma_commit(&bar);
    }
    {
      // C rows times 1/m^2 (W / m = (C / m) V / m) -> the W groups' left operands;
      // the first two blocks load while V is formed
      constexpr int kEarly = NPB < 2 ? NPB : 2;
      const float* crec = rec + 2 * r * r;
      RowLd cl[kEarly];
#pragma unroll
      for (int pb = 0; pb < kEarly; ++pb) row_issue(cl[pb], crec + pb * 32 * r, lane, P - 32 * pb, r);
      ok &= product_wait(&bar, phase, d.wlim);
      tc::tmem_ld32(tmine, t);
      if (keep) store_op(opq + kOpV * kOpFloats, t, lane);
      put_row<true>(S0, w, lane, t);                    // C(V): S0 is free once V has landed
      unsigned char* cs = smem + (size_t)(1 + w / kCpg) * kSlot;
#pragma unroll
      for (int pb = 0; pb < NPB; ++pb) {
        if (pb < kEarly) {
          row_finish(t, cl[pb], 32 * pb + lane < P, im2);
        } else if (32 * pb < P) {
          RowLd l;
          row_issue(l, crec + pb * 32 * r, lane, P - 32 * pb, r);
          row_finish(t, l, 32 * pb + lane < P, im2);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) t[j] = 0.f;      // rows past P (P = 96 in four blocks)
        }
        put_row_at(cs, 32 * NPB * (w % kCpg) + 32 * pb + lane, t);
      }
    }
    operands_ready();
    if (tid == 0) {
      tc::fence_after_sync();
#pragma unroll
      for (int g = 0; g < NPB; ++g)
        mma3(tmem + (uint32_t)(g * kGroupCols), a1 + (uint32_t)g * kSlot, false, a0 + (uint32_t)(g * kCpg) * 2048u,
             true, kGroupCols, false);
      tc::mma_commit(&bar);
    }
    ok &= product_wait(&bar, phase, d.wlim);
    const bool failed = __syncthreads_or(!ok) != 0;
    if (valid && lane == 0) {
      invs_out[q] = invs;
      if (failed) status[q] |= 2 << 4;                  // bits 4-5: this kernel's product wait
    }
    // W group g: TMEM lane 32w + lane is row p = 32 (w % NPB) + lane of local chunk g kCpg + w / NPB
#pragma unroll
    for (int g = 0; g < NPB; ++g) {
      const int lc = w / NPB;
      tc::tmem_ld32(tmem + ((uint32_t)(32 * w) << 16) + (uint32_t)(g * kGroupCols + 32 * lc), t);
      const long long qq = q0 + g * kCpg + lc;
      const int p = 32 * (w % NPB) + lane;
      if (qq < nq && p < P) store_wm_row(wm_out + (size_t)qq * P * r * 4, t, p, P, r, failed);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (w == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kOpsCols);
  }
}

// ---------------------------------------------------------------------------
// backward: the chain rule through W = Cn Li^T A^K Li from the operators the
// forward kept (Li^T, A, A^K, U, V, S), four chunks per CTA, every r x r product
// batched as in the forward.  Same algebra as wpc::k_bwd_chunk_s:
//   dV = C^T dW' / m^2,  m dCn = dW' V^T,  dU = Li dV,  dLi = U dV^T + A^K^T dU,
//   dA^K = dU Li^T,  dA = dA^K A^T + A^T dA^K (K = 2),  dMn = kk dA S,
//   dS + dS^T = kk (Mn^T dA + dA^T Mn),  dLi += Li (dS + dS^T),
//   Pm = tril(-tril(dLi) Li^T),  P' = (Pm + tril(Pm, -1)^T) / 2,
//   dGn = sym(Li^T P' Li).
// Transposes never happen in registers: an operand is written in the R or C
// arrangement that gives the tensor core the orientation it needs, and the
// symmetrisations are sums of two products into one accumulator.  Two TMEM
// regions of 128 columns let two independent products share a round trip.
// Each step's global rows are loaded before the previous step's product wait.
// Persistent like the forward.
// ---------------------------------------------------------------------------
constexpr uint32_t kBwdCols = 256;
constexpr int kBwdSlots = 4;

// rows [0, nrows) of an nrows x r row-major record block <- row `lane` of v * scale,
// through the warp's staging buffer and one bulk copy (the rows are contiguous)
__device__ __forceinline__ void st_rec_async(float* dst, const float (&v)[32], int nrows, int r, float scale,
                                             float* stg, int lane) {
  if (nrows <= 0) return;
  if (nrows > 32) nrows = 32;
  stage_acquire(lane);
  if (lane < nrows) {
    float4* p = reinterpret_cast<float4*>(stg + lane * r);
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (4 * k < r)
        p[k] = make_float4(v[4 * k] * scale, v[4 * k + 1] * scale, v[4 * k + 2] * scale, v[4 * k + 3] * scale);
  }
  stage_release(dst, stg, (uint32_t)(nrows * r) * 4u, lane);
}

__device__ __forceinline__ float dot32(const float (&a)[32], const float (&b)[32]) {
  float s0 = 0.f, s1 = 0.f;
#pragma unroll
  for (int j = 0; j < 32; j += 2) {
    s0 = fmaf(a[j], b[j], s0);
    s1 = fmaf(a[j + 1], b[j + 1], s1);
  }
  return s0 + s1;
}

// everything chunk q's backward reads, on its way to L2
__device__ __forceinline__ void bwd_prefetch(const Dims& d, const float* stats, const float* ops, const float* dwraw,
                                             long long q, int lane) {
  prefetch_l2(ops + q * (long long)(kNumOps * kOpFloats), kNumOps * kOpFloats * 4, lane);
  prefetch_l2(stats + q * d.SW, d.SW * 4, lane);
  prefetch_l2(dwraw + q * (long long)d.P * d.r, d.P * d.r * 4, lane);
}

__global__ void __launch_bounds__(kOpsThreads, 2) k_bwd_ops_tc(Dims d, const float* __restrict__ gamma_p,
                                                               const float* __restrict__ stats,
                                                               const unsigned long long* __restrict__ cmax,
                                                               const float* __restrict__ invs_in,
                                                               const float* __restrict__ ops,
                                                               const float* __restrict__ dwraw,
                                                               float* __restrict__ dstats,
                                                               float* __restrict__ dmpart,
                                                               float* __restrict__ dgpart, int* __restrict__ status) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ uint64_t bar, bar2;   // products into R0 (thread 0) and into R1 (thread 32)
  __shared__ uint32_t tmem_slot;
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  const long long nq = (long long)d.B * d.H * d.C;
  const long long ngroups = (nq + 3) / 4;
  const int r = d.r, P = d.P;
  bwd_prefetch(d, stats, ops, dwraw, (long long)blockIdx.x * 4 + w < nq ? (long long)blockIdx.x * 4 + w : nq - 1,
               lane);
  unsigned char* X = smem;
  unsigned char* Y = smem + kSlot;
  unsigned char* Z = smem + 2 * kSlot;
  unsigned char* Wt = smem + 3 * kSlot;
  const uint32_t aX = tc::smem_u32(X), aY = aX + kSlot, aZ = aX + 2 * kSlot, aW = aX + 3 * kSlot;
  float* stg = reinterpret_cast<float*>(smem + (size_t)kBwdSlots * kSlot + (size_t)w * kStageBytes);
  // this warp's two fp32 tiles for record blocks (C and dW' blocks, then M, then G):
  // cp.async copies of whole 32 x 32 blocks (coalesced; row `lane` loads would touch
  // 32 lines per instruction), read back a row per lane without bank conflicts
  float* TC = reinterpret_cast<float*>(smem + (size_t)kBwdSlots * kSlot + 4 * kStageBytes + (size_t)w * 8192);
  float* TW = TC + 1024;

  if (w == 0) tc::tmem_alloc(&tmem_slot, kBwdCols);
  if (tid == 0) {
    tc::mbar_init(&bar, 1);
    tc::mbar_init(&bar2, 1);
    tc::mbar_fence_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t R0 = tmem_slot, R1 = tmem_slot + 128u;
  const uint32_t mine = ((uint32_t)(32 * w) << 16) + (uint32_t)(32 * w);   // this warp's diagonal block
  const float gam = *gamma_p;
  const float gs = fminf(fmaxf(gam, 1.f), 1.5f);
  const bool gpass = gam >= 1.f && gam <= 1.5f;       // the clamp passes gradients inclusively
  const int npb = (P + 31) >> 5;
  uint32_t phase = 0, phase2 = 0;

#pragma unroll 1
  for (long long gi = blockIdx.x; gi < ngroups; gi += gridDim.x) {
    const bool valid = gi * 4 + w < nq;
    const long long q = valid ? gi * 4 + w : nq - 1;   // a spare warp stores nothing
    const float* rec = stats + q * d.SW;
    const float* opq = ops + q * (long long)(kNumOps * kOpFloats);
    const float* dwq = dwraw + q * (long long)P * r;
    const float* crec = rec + 2 * r * r;
    float* drec = dstats + q * d.SW;
    // block 0's C and dW' rows (the tiles' last reader was this warp: sync first)
    __syncwarp();
    wpc::cp_tile_async(TC, crec, P < 32 ? P : 32, r, lane);
    wpc::cp_tile_async(TW, dwq, P < 32 ? P : 32, r, lane);
    wpc::cp_async_commit();
    if (gi + gridDim.x < ngroups) {   // what the next group's first step reads: V, the C rows, dW'
      long long qn = (gi + gridDim.x) * 4 + w;
      qn = qn < nq ? qn : nq - 1;
      prefetch_l2(ops + qn * (long long)(kNumOps * kOpFloats) + kOpV * kOpFloats, kOpFloats * 4, lane);
      prefetch_l2(stats + qn * d.SW + 2 * r * r, P * r * 4, lane);
      prefetch_l2(dwraw + qn * (long long)P * r, P * r * 4, lane);
    }
    bool ok = true;
    const ChunkId id = wpc::chunk_id(d, q);
    const float m = wpc::series_norm(cmax, id, d.C, lane), im = 1.f / m, im2 = im * im;
    const float kk = gs * invs_in[q];
    float t[32], u[32], a1[32], a2[32];   // a1, a2: rows loaded ahead, across the product waits

    // ---- P blocks: dV = sum_pb C_pb^T dW'_pb / m^2 (R0), TY_pb = dW'_pb V^T (R1) ----
    float dmc = 0.f;
    ld_op_row(t, opq + kOpV * kOpFloats, lane);
    put_row<false>(Wt, w, lane, t);                     // R(V): the right operand V^T
#pragma unroll 1
    for (int pb = 0; pb < npb; ++pb) {
      wpc::cp_async_wait<0>();
      __syncwarp();
      wpc::ld_row(a1, TC, lane);                         // C rows (raw; zero past P)
      wpc::ld_row(a2, TW, lane);                         // dW' rows
#pragma unroll
      for (int j = 0; j < 32; ++j) t[j] = a1[j] * im2;
      put_row<true>(X, w, lane, t);                     // C(C_pb / m^2): the left operand C_pb^T / m^2
      put_row_rc(Z, Y, w, lane, a2);                    // R(dW'_pb): the left operand dW'_pb; C: the right
      operands_ready();
      if (tid == 0) {
        tc::fence_after_sync();
        mma3(R0, aX, true, aY, true, 128, pb > 0);
        tc::mma_commit(&bar);
      } else if (tid == 32) {
        tc::fence_after_sync();
        mma3(R1, aZ, false, aW, false, 128, false);
        tc::mma_commit(&bar2);
      }
      if (pb + 1 < npb) {
        const int nr = P - 32 * (pb + 1) < 32 ? P - 32 * (pb + 1) : 32;
        wpc::cp_tile_async(TC, crec + (pb + 1) * 32 * r, nr, r, lane);   // read before the block barrier
        wpc::cp_tile_async(TW, dwq + (pb + 1) * 32 * r, nr, r, lane);
        wpc::cp_async_commit();
      } else {
        ld_op_row(a2, opq + kOpLi * kOpFloats, lane);   // for the next step: Li^T
        ld_op_row(u, opq + kOpU * kOpFloats, lane);     //   and U
      }
      ok &= product_wait(&bar, phase, d.wlim);
      ok &= product_wait(&bar2, phase2, d.wlim);
      tc::tmem_ld32(R1 + mine, t);                      // TY rows p = 32 pb + lane
      if (valid) st_rec_async(drec + 2 * r * r + pb * 32 * r, t, P - 32 * pb, r, im2, stg, lane);   // dCn / m
      dmc += dot32(t, a1);                              // <TY, C> = m^2 <dCn, Cn>
    }
    tc::tmem_ld32(R0 + mine, t);                        // dV
    ld_op_row(a1, opq + kOpV * kOpFloats, lane);
    const float dmq = dot32(a1, t);                     // <V, dV> = <W, dW>
    // ---- dU = Li dV (R0), dLi = U dV^T (R1) ----
    float dli[32];
    touch32(a2);
    touch32(u);
    put_row<true>(Wt, w, lane, a2);                     // C(Li^T): the left operand Li, the right operand Li^T
    put_row_rc(Z, Y, w, lane, t);                       // R(dV): the right operand dV^T; C(dV)
    put_row<false>(X, w, lane, u);                      // R(U)
    operands_ready();
    if (tid == 0) {
      tc::fence_after_sync();
      mma3(R0, aW, true, aY, true, 128, false);
      tc::mma_commit(&bar);
    } else if (tid == 32) {
      tc::fence_after_sync();
      mma3(R1, aX, false, aZ, false, 128, false);
      tc::mma_commit(&bar2);
    }
    ld_op_row(a1, opq + kOpAK * kOpFloats, lane);       // for the next step: A^K
    ld_op_row(a2, opq + kOpA * kOpFloats, lane);        //   and A
    ok &= product_wait(&bar, phase, d.wlim);
    ok &= product_wait(&bar2, phase2, d.wlim);
    tc::tmem_ld32(R0 + mine, t);                        // dU
    tc::tmem_ld32(R1 + mine, dli);
    // ---- dAK = dU Li^T (R0), dLi += AK^T dU (R1) ----
    touch32(a1);
    put_row<true>(X, w, lane, a1);                      // C(AK): the left operand AK^T
    put_row_rc(Y, Z, w, lane, t);                       // R(dU), C(dU)
    operands_ready();
    if (tid == 0) {
      tc::fence_after_sync();
      mma3(R0, aY, false, aW, true, 128, false);
      tc::mma_commit(&bar);
    } else if (tid == 32) {
      tc::fence_after_sync();
      mma3(R1, aX, true, aZ, true, 128, false);
      tc::mma_commit(&bar2);
    }
    ld_op_row(a1, opq + kOpS * kOpFloats, lane);        // for the step after: S
    wpc::cp_tile_async(TC, rec + r * r, r, r, lane);    //   and M (TC was last read before a block barrier)
    wpc::cp_async_commit();
    ok &= product_wait(&bar, phase, d.wlim);
    ok &= product_wait(&bar2, phase2, d.wlim);
    tc::tmem_ld32(R0 + mine, t);                        // dAK
    tc::tmem_ld32(R1 + mine, u);
#pragma unroll
    for (int j = 0; j < 32; ++j) dli[j] += u[j];
    // ---- dA (K = 2: dAK A^T + A^T dAK in R0; K = 1: dAK; K = 0: zero) ----
    touch32(a2);
    if (d.K == 2) {
      put_row_rc(X, Y, w, lane, a2);                    // R(A): the right operand A^T; C(A): the left operand A^T
      put_row_rc(Z, Wt, w, lane, t);                    // R(dAK), C(dAK)
      operands_ready();
      if (tid == 0) {
        tc::fence_after_sync();
        mma3(R0, aZ, false, aX, false, 128, false);
        mma3(R0, aY, true, aW, true, 128, true);
        tc::mma_commit(&bar);
      }
      ok &= product_wait(&bar, phase, d.wlim);
      tc::tmem_ld32(R0 + mine, t);
    } else if (d.K == 0) {
#pragma unroll
      for (int j = 0; j < 32; ++j) t[j] = 0.f;
    }
    const float dg = dot32(t, a2);                      // <dA, A>
    // ---- dMn = kk dA S (R0), dS + dS^T = kk (Mn^T dA + dA^T Mn) (R1) ----
    touch32(a1);
    put_row<true>(X, w, lane, a1);                      // C(S)
    wpc::cp_async_wait<0>();
    __syncwarp();
    wpc::ld_row(a2, TC, lane);                          // Mn rows
#pragma unroll
    for (int j = 0; j < 32; ++j) a2[j] *= im2;
    put_row<true>(Y, w, lane, a2);                      // C(Mn): the left operand Mn^T, the right operand Mn
    put_row_rc(Z, Wt, w, lane, t);                      // R(dA); C(dA): the left operand dA^T, the right operand dA
    operands_ready();
    if (tid == 0) {
      tc::fence_after_sync();
      mma3(R0, aZ, false, aX, true, 128, false);
      tc::mma_commit(&bar);
    } else if (tid == 32) {
      tc::fence_after_sync();
      mma3(R1, aY, true, aW, true, 128, false);
      mma3(R1, aW, true, aY, true, 128, true);
      tc::mma_commit(&bar2);
    }
    ld_op_row(a1, opq + kOpLi * kOpFloats, lane);       // for the next steps: Li^T
    ok &= product_wait(&bar, phase, d.wlim);
    ok &= product_wait(&bar2, phase2, d.wlim);
    tc::tmem_ld32(R0 + mine, t);
#pragma unroll
    for (int j = 0; j < 32; ++j) t[j] *= kk;            // dMn
    if (valid) st_rec_async(drec + r * r, t, r, r, im2, stg, lane);
    const float dmm = dot32(t, a2);
    tc::tmem_ld32(R1 + mine, t);
#pragma unroll
    for (int j = 0; j < 32; ++j) t[j] *= kk;            // dS + dS^T
    // ---- dLi += Li (dS + dS^T) (R0) ----
    touch32(a1);
    put_row_rc(Z, Y, w, lane, a1);                      // R(Li^T), for the steps after; C(Li^T)
    put_row<true>(X, w, lane, t);                       // C(dS + dS^T)
    operands_ready();
    if (tid == 0) {
      tc::fence_after_sync();
      mma3(R0, aY, true, aX, true, 128, false);
      tc::mma_commit(&bar);
    }
    wpc::cp_tile_async(TW, rec, r, r, lane);            // for the end: G
    wpc::cp_async_commit();
    ok &= product_wait(&bar, phase, d.wlim);
    tc::tmem_ld32(R0 + mine, t);
#pragma unroll
    for (int j = 0; j < 32; ++j) dli[j] = (j > lane) ? 0.f : dli[j] + t[j];   // only tril(dLi) reaches L
    // ---- Pm = tril(-tril(dLi) Li^T) (R0) ----
    put_row<false>(X, w, lane, dli);                    // R(tril dLi)
    operands_ready();
    if (tid == 0) {
      tc::fence_after_sync();
      mma3(R0, aX, false, aY, true, 128, false);
      tc::mma_commit(&bar);
    }
    ok &= product_wait(&bar, phase, d.wlim);
    tc::tmem_ld32(R0 + mine, t);
    // P' = (L'' + L''^T) / 2 with L'' = tril(Pm), its diagonal halved
#pragma unroll
    for (int j = 0; j < 32; ++j) t[j] = (j < lane) ? -t[j] : (j == lane ? -0.5f * t[j] : 0.f);
    // ---- T1 = P' Li = (L'' Li + L''^T Li) / 2 (R0) ----
    put_row_rc(X, Y, w, lane, t);                       // R(L''); C(L''): the left operand L''^T
    operands_ready();
    if (tid == 0) {
      tc::fence_after_sync();
      mma3(R0, aX, false, aZ, false, 128, false);
      mma3(R0, aY, true, aZ, false, 128, true);
      tc::mma_commit(&bar);
    }
    ok &= product_wait(&bar, phase, d.wlim);
    tc::tmem_ld32(R0 + mine, t);
#pragma unroll
    for (int j = 0; j < 32; ++j) t[j] *= 0.5f;
    // ---- sym(dGn) = (Li^T T1 + T1^T Li) / 2 (R0) ----
    put_row<true>(X, w, lane, t);                       // C(T1): the right operand T1, the left operand T1^T
    operands_ready();
    if (tid == 0) {
      tc::fence_after_sync();
      mma3(R0, aZ, false, aX, true, 128, false);
      mma3(R0, aX, true, aZ, false, 128, true);
      tc::mma_commit(&bar);
    }
    ok &= product_wait(&bar, phase, d.wlim);
    tc::tmem_ld32(R0 + mine, t);
    wpc::cp_async_wait<0>();
    __syncwarp();
    wpc::ld_row(a2, TW, lane);                          // G rows and columns (zero past r)
    wpc::ld_col<32>(a1, TW, lane);
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      t[j] *= 0.5f;
      u[j] = 0.5f * (a2[j] + a1[j]) * im2;              // sym(G) / m^2 (zero past r)
    }
    const float dmg = dot32(t, u);
    const bool failed = __syncthreads_or(!ok) != 0;
    if (valid) st_rec_async(drec, t, r, r, im2, stg, lane);   // dGn / m^2
    const float tot = wpc::warp_sum32(2.f * dmg + 2.f * dmm + dmc * im2 + dmq);
    const float dgs = wpc::warp_sum32(dg);
    if (valid && lane == 0) {
      dmpart[q] = failed ? __int_as_float(0x7fc00000) : -tot / m;
      dgpart[q] = gpass ? dgs / gs : 0.f;
      if (failed) status[q] |= 2 << 4;                  // bits 4-5: this kernel's product wait
    }
  }
  if (lane == 0) tc::bulk_wait();   // the records are written before the kernel ends
  tc::fence_before_sync();
  __syncthreads();
  if (w == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(R0, kBwdCols);
  }
}

}  // namespace otc

// r <= 32 with r % 16 == 0 (the readout operand's K steps) and P <= 128
bool ops_tc_ok(const Dims& d) { return d.r <= 32 && d.r % 16 == 0 && d.P <= 128; }
// and power_K <= 2 for the backward (its Horner step is one batched pair of products)
bool bwd_ops_tc_ok(const Dims& d) { return ops_tc_ok(d) && d.K <= 2; }

// lit: room for every chunk's Li^T (32 x 32 fp32)
cudaError_t launch_fwd_ops_tc(const Dims& d, const float* gamma, const float* stats, const unsigned long long* cmax,
                              float* invs, int* flags, float* lit, float* ops, unsigned char* wm, int* status,
                              cudaStream_t st) {
  const long long nq = (long long)d.B * d.H * d.C;
  if (nq == 0) return cudaSuccess;
  const bool r16 = d.r <= 16;   // factored inside the operator kernel
  if (!r16) {
    const unsigned fgrid = (unsigned)((nq + otc::kFac32Warps - 1) / otc::kFac32Warps);
    otc::k_factor32<false><<<fgrid, otc::kFac32Warps * 32, 0, st>>>(d, stats, cmax, lit, flags);
    const cudaError_t e0 = cudaGetLastError();
    if (e0 != cudaSuccess) return e0;
  }
  const int npb = otc::ops_npb(d.P);
  const size_t smem = (size_t)otc::ops_slots(npb) * otc::kSlot;
  Dims dd = d;
  void* args[] = {&dd, (void*)&gamma, (void*)&stats, (void*)&cmax, (void*)&invs, (void*)&flags, (void*)&lit, (void*)&ops,
                  (void*)&wm, (void*)&status};
  const void* fn = npb == 1 ? (r16 ? reinterpret_cast<const void*>(otc::k_fwd_ops_tc<1, true>)
                                   : reinterpret_cast<const void*>(otc::k_fwd_ops_tc<1>))
                   : npb == 2 ? (r16 ? reinterpret_cast<const void*>(otc::k_fwd_ops_tc<2, true>)
                                     : reinterpret_cast<const void*>(otc::k_fwd_ops_tc<2>))
                              : reinterpret_cast<const void*>(otc::k_fwd_ops_tc<4>);
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  unsigned grid = 0;
  if ((e = otc::persistent_grid(fn, smem, 512 / (int)otc::kOpsCols, (nq + 3) / 4, &grid)) != cudaSuccess) return e;
  e = cudaLaunchKernel(fn, dim3(grid), dim3(otc::kOpsThreads), args, smem, st);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t launch_bwd_ops_tc(const Dims& d, const float* gamma, const float* stats, const unsigned long long* cmax,
                              const float* invs, const float* ops, const float* dwraw, float* dstats, float* dmpart,
                              float* dgpart, int* status, cudaStream_t st) {
  const long long nq = (long long)d.B * d.H * d.C;
  if (nq == 0) return cudaSuccess;
  const size_t smem = (size_t)otc::kBwdSlots * otc::kSlot + 4 * otc::kStageBytes + 4 * 8192;
  Dims dd = d;
  void* args[] = {&dd, (void*)&gamma, (void*)&stats, (void*)&cmax, (void*)&invs, (void*)&ops, (void*)&dwraw,
                  (void*)&dstats, (void*)&dmpart, (void*)&dgpart, (void*)&status};
  const void* fn = reinterpret_cast<const void*>(otc::k_bwd_ops_tc);
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  unsigned grid = 0;
  if ((e = otc::persistent_grid(fn, smem, 512 / (int)otc::kBwdCols, (nq + 3) / 4, &grid)) != cudaSuccess) return e;
  e = cudaLaunchKernel(fn, dim3(grid), dim3(otc::kOpsThreads), args, smem, st);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace ska
