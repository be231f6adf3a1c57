// ska_capi.cu -- extern "C" entry points of libska_b200.so (declared in
// include/ska_b200.h): argument validation, workspace layout, dispatch.
#include "../../include/ska_b200.h"
#include "ska_common.cuh"
#include "ska_tc.cuh"

#include <atomic>
#include <cmath>
#include <vector>

namespace ska {
template <typename T>
cudaError_t launch_fwd(const Dims&, const In&, const In&, const In&, const float*, const Out&,
                       const SavedLayout&, char*, cudaStream_t, bool, bool);
template <typename T>
cudaError_t launch_bwd(const Dims&, const In&, const In&, const In&, const float*, const In&,
                       const SavedLayout&, const char*, const ScratchLayout&, char*, const Out&, const Out&,
                       const Out&, float*, cudaStream_t);
size_t smem_fwd_stats(const Dims&);
size_t smem_fwd_chunk(const Dims&);
size_t smem_bwd_chunk(const Dims&);
size_t smem_bwd_tok(const Dims&);
bool warp_path_ok(const Dims&);
bool quad_path_ok(const Dims&);
bool ops_tc_ok(const Dims&);
bool bwd_ops_tc_ok(const Dims&);
size_t smem_fwd_chunk_w(const Dims&);
size_t smem_bwd_chunk_w(const Dims&);
namespace tc {
bool stats_tc_ok(const Dims& d, const In& z, const In& v);
bool stats_scan_tc_ok(const Dims& d, const In& z, const In& v);
}
template <typename IO>
bool fwd_tc_readout(const Dims& d, const In& zq, const Out& y);
template <typename IO>
void bwd_tc_paths(const Dims& d, const In& z, const In& zq, const In& v, const In& dy, const Out& dz,
                  const Out& dzq, const Out& dv, bool* full, bool* tok);
struct StateLayout {
  size_t G, M, C, zlast, maxnorm, flags, total;
};
StateLayout state_layout(long long B, long long H, long long r, long long P);
cudaError_t launch_state_init(const Dims& d, char* state, const StateLayout& L, cudaStream_t st);
template <typename IO>
cudaError_t launch_prefill_state(const Dims& d, const In& z, const In& v, const float* stats,
                                 const unsigned long long* cmax, char* state, const StateLayout& L, cudaStream_t st);
template <typename IO>
cudaError_t launch_step(const Dims& d, const In& z, const In& zq, const In& v, const float* gamma, const Out& y,
                        char* state, const StateLayout& L, cudaStream_t st);
}  // namespace ska

namespace {

using ska::Dims;

// polls before a tensor-core kernel's first wait of a role gives up (ska_set_wait_limit)
std::atomic<uint32_t> g_wait_limit{ska::tc::kWaitLimit};

int make_dims(const SkaShape* s, Dims* d) {
  if (!s) return SKA_ERR_NULL;
  if (s->B < 0 || s->T < 1 || s->H < 1 || s->r < 1 || s->P < 1 || s->chunk_size < 1 || s->power_K < 0)
    return SKA_ERR_SHAPE;
  if (s->r > ska::kMaxRank || s->P > ska::kMaxP || s->chunk_size > ska::kMaxChunk ||
      s->power_K > ska::kMaxPowerK)
    return SKA_ERR_UNSUPPORTED;
  const long long C = (s->T + s->chunk_size - 1) / s->chunk_size;
  // grid limits: (C, H, B) and (SW/256, B*H)
  if (s->H > 65535 || s->B > 65535 || s->B * s->H > 65535 || C > 0x7fffffffLL || s->T > 0x7fffffffLL)
    return SKA_ERR_UNSUPPORTED;
  if (s->strategy != SKA_STRATEGY_STANDARD && s->strategy != SKA_STRATEGY_DECAY) return SKA_ERR_STRATEGY;
  if (s->strategy == SKA_STRATEGY_DECAY && !std::isfinite(s->decay_alpha)) return SKA_ERR_STRATEGY;
  d->B = (int)s->B;
  d->T = (int)s->T;
  d->H = (int)s->H;
  d->r = (int)s->r;
  d->P = (int)s->P;
  d->CS = (int)s->chunk_size;
  d->C = (int)C;
  d->K = s->power_K;
  d->decay = s->strategy == SKA_STRATEGY_DECAY ? 1 : 0;
  d->ridge = s->ridge_eps;
  d->alpha = d->decay ? s->decay_alpha : 1.f;
  d->SW = 2 * d->r * d->r + d->P * d->r;
  d->wlim = g_wait_limit.load(std::memory_order_relaxed);
  // every kernel's shared-memory tile set must fit one sm_100a CTA (227 KB opt-in)
  const size_t kMaxSmem = 232448;
  if (ska::smem_fwd_stats(*d) > kMaxSmem || ska::smem_bwd_tok(*d) > kMaxSmem) return SKA_ERR_UNSUPPORTED;
  if (ska::warp_path_ok(*d)) {
    if (ska::smem_fwd_chunk_w(*d) == 0 || ska::smem_bwd_chunk_w(*d) == 0) return SKA_ERR_UNSUPPORTED;
  } else if (ska::smem_fwd_chunk(*d) > kMaxSmem || ska::smem_bwd_chunk(*d) > kMaxSmem) {
    return SKA_ERR_UNSUPPORTED;
  }
  return SKA_OK;
}

int elem_size(int dtype) {
  switch (dtype) {
    case SKA_DTYPE_F32: return 4;
    case SKA_DTYPE_BF16: return 2;
    default: return 0;
  }
}

int check_tensor(const SkaTensor* t, int esize, bool needed, ska::In* out) {
  if (!t) return SKA_ERR_NULL;
  if (needed && !t->data) return SKA_ERR_NULL;
  if (reinterpret_cast<uintptr_t>(t->data) % (uintptr_t)esize) return SKA_ERR_ALIGN;
  out->p = t->data;
  out->sb = t->stride_b;
  out->st = t->stride_t;
  out->sh = t->stride_h;
  return SKA_OK;
}

int check_out(const SkaTensor* t, int esize, bool needed, ska::Out* out) {
  ska::In tmp{};
  const int rc = check_tensor(t, esize, needed, &tmp);
  if (rc) return rc;
  out->p = t->data;
  out->sb = t->stride_b;
  out->st = t->stride_t;
  out->sh = t->stride_h;
  return SKA_OK;
}

}  // namespace

namespace ska {
ProfileEvents* profile_events() {
  static ProfileEvents p{};
  return &p;
}
}  // namespace ska

extern "C" {

int ska_abi_version(void) { return SKA_ABI_VERSION; }

int ska_set_profile_events(void* const* events, int count) {
  ska::ProfileEvents* p = ska::profile_events();
  if (!events) {
    p->on = false;
    return SKA_OK;
  }
  if (count < SKA_PROFILE_EVENTS) return SKA_ERR_SHAPE;
  for (int i = 0; i < SKA_PROFILE_EVENTS; ++i) {
    if (!events[i]) return SKA_ERR_NULL;
    p->ev[i] = static_cast<cudaEvent_t>(events[i]);
  }
  p->on = true;
  return SKA_OK;
}

int ska_kernel_path(const SkaShape* shape, int io_dtype, const SkaTensor* z, const SkaTensor* v) {
  Dims d{};
  int rc = make_dims(shape, &d);
  if (rc) return rc;
  if (io_dtype == SKA_DTYPE_BF16_Y32) io_dtype = SKA_DTYPE_BF16;   // the same kernels
  const int es = elem_size(io_dtype);
  if (!es) return SKA_ERR_DTYPE;
  ska::In iz{}, iv{};
  if ((rc = check_tensor(z, es, true, &iz)) || (rc = check_tensor(v, es, true, &iv))) return rc;
  int mask = 0;
  if (io_dtype == SKA_DTYPE_BF16 && ska::tc::stats_tc_ok(d, iz, iv)) mask |= SKA_PATH_TC_STATS;
  if (io_dtype == SKA_DTYPE_BF16 && ska::tc::stats_scan_tc_ok(d, iz, iv)) mask |= SKA_PATH_FUSED_SCAN;
  if (ska::warp_path_ok(d)) mask |= SKA_PATH_WARP_CHUNK;
  if (io_dtype == SKA_DTYPE_BF16 && ska::quad_path_ok(d)) {   // zq and y assumed laid out like z and v
    const ska::Out yv{const_cast<void*>(iv.p), iv.sb, iv.st, iv.sh};
    if (ska::fwd_tc_readout<__nv_bfloat16>(d, iz, yv)) mask |= SKA_PATH_QUAD_CHUNK;
  }
  if (io_dtype == SKA_DTYPE_BF16) {   // y assumed laid out like v
    const ska::Out yv{const_cast<void*>(iv.p), iv.sb, iv.st, iv.sh};
    if (ska::fwd_tc_readout<__nv_bfloat16>(d, iz, yv)) {
      mask |= SKA_PATH_TC_READOUT_FWD;
      if (ska::warp_path_ok(d) && ska::ops_tc_ok(d)) mask |= SKA_PATH_TC_CHUNK_FWD;
    }
  }
  if (io_dtype == SKA_DTYPE_BF16) {   // gradients and zq, dy assumed laid out like z and v
    const ska::Out gz{const_cast<void*>(iz.p), iz.sb, iz.st, iz.sh}, gv{const_cast<void*>(iv.p), iv.sb, iv.st, iv.sh};
    bool full = false, tok = false;
    ska::bwd_tc_paths<__nv_bfloat16>(d, iz, iz, iv, iv, gz, gz, gv, &full, &tok);
    if (tok) mask |= SKA_PATH_TC_TOKEN_BWD;
    if (full) mask |= SKA_PATH_TC_READOUT_BWD;
    if (full && ska::warp_path_ok(d) && ska::bwd_ops_tc_ok(d)) mask |= SKA_PATH_TC_CHUNK_BWD;
    if (full && !ska::warp_path_ok(d)) mask |= SKA_PATH_QUAD_CHUNK_BWD;
  }
  return mask;
}

const char* ska_status_string(int code) {
  switch (code) {
    case SKA_OK: return "ok";
    case SKA_ERR_NULL: return "a required pointer is NULL";
    case SKA_ERR_SHAPE: return "invalid shape (need B>=0, T>=1, H>=1, r>=1, P>=1, chunk_size>=1, power_K>=0)";
    case SKA_ERR_UNSUPPORTED: return "unsupported size (r<=64, P<=128, chunk_size<=256, power_K<=8, B*H<=65535)";
    case SKA_ERR_DTYPE: return "unknown io dtype";
    case SKA_ERR_WORKSPACE: return "saved or scratch buffer too small";
    case SKA_ERR_ALIGN: return "misaligned pointer";
    case SKA_ERR_LAUNCH: return "CUDA kernel launch failed";
    case SKA_ERR_STRATEGY: return "unknown chunk strategy or non-finite decay_alpha";
    case SKA_ERR_TIMEOUT: return "a tensor-core kernel's bounded wait expired (its chunks' outputs are NaN)";
    default: return "unknown status";
  }
}

int ska_set_wait_limit(uint32_t polls) {
  g_wait_limit.store(polls == 0xFFFFFFFFu ? ska::tc::kWaitLimit : polls, std::memory_order_relaxed);
  return SKA_OK;
}

int ska_check_status(const SkaShape* shape, const void* saved, size_t saved_bytes, const void* scratch,
                     size_t scratch_bytes, void* stream, int64_t* first_bad, int* code) {
  Dims d{};
  int rc = make_dims(shape, &d);
  if (rc) return rc;
  if (first_bad) *first_bad = -1;
  if (code) *code = 0;
  const size_t n = (size_t)d.B * d.H * d.C;
  if (n == 0) return SKA_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  std::vector<int> host(n);
  // forward entries first, then backward (bits 0-1 readout gradient, 2-3 token kernel)
  for (int part = 0; part < 2; ++part) {
    const char* base = static_cast<const char*>(part ? scratch : saved);
    if (!base) continue;
    if (reinterpret_cast<uintptr_t>(base) % 256) return SKA_ERR_ALIGN;
    const size_t off = part ? ska::scratch_layout(d.B, d.H, d.C, d.SW, d.r, d.P).status
                            : ska::saved_layout(d.B, d.H, d.C, d.SW, d.r, d.P).status;
    const size_t have = part ? scratch_bytes : saved_bytes;
    if (have < off + n * sizeof(int)) return SKA_ERR_WORKSPACE;
    if (cudaMemcpyAsync(host.data(), base + off, n * sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
      return SKA_ERR_LAUNCH;
    for (size_t i = 0; i < n; ++i) {
      if (host[i] != 0) {
        if (first_bad) *first_bad = (int64_t)i;
        if (code) *code = part ? SKA_STATUS_BWD_BASE + host[i] : host[i];
        return SKA_ERR_TIMEOUT;
      }
    }
  }
  return SKA_OK;
}

int ska_workspace_size(const SkaShape* shape, size_t* saved_bytes, size_t* scratch_bytes) {
  Dims d{};
  const int rc = make_dims(shape, &d);
  if (rc) return rc;
  if (saved_bytes) *saved_bytes = ska::saved_layout(d.B, d.H, d.C, d.SW, d.r, d.P).total;
  if (scratch_bytes) *scratch_bytes = ska::scratch_layout(d.B, d.H, d.C, d.SW, d.r, d.P).total;
  return SKA_OK;
}

int ska_forward_workspace_size(const SkaShape* shape, size_t* saved_bytes) {
  Dims d{};
  const int rc = make_dims(shape, &d);
  if (rc) return rc;
  if (saved_bytes) *saved_bytes = ska::saved_layout(d.B, d.H, d.C, d.SW, d.r, d.P).fwd;
  return SKA_OK;
}

int ska_fwd(const SkaShape* shape, int io_dtype, const SkaTensor* z, const SkaTensor* zq, const SkaTensor* v,
            const float* gamma, const SkaTensor* y, void* saved, size_t saved_bytes, void* stream) {
  Dims d{};
  int rc = make_dims(shape, &d);
  if (rc) return rc;
  // SKA_DTYPE_BF16_Y32: bf16 z, zq, v with an fp32 y
  const bool y32 = io_dtype == SKA_DTYPE_BF16_Y32;
  const int es = elem_size(y32 ? SKA_DTYPE_BF16 : io_dtype);
  if (!es) return SKA_ERR_DTYPE;
  const bool work = d.B > 0;
  ska::In iz{}, izq{}, iv{};
  ska::Out oy{};
  if ((rc = check_tensor(z, es, work, &iz)) || (rc = check_tensor(zq, es, work, &izq)) ||
      (rc = check_tensor(v, es, work, &iv)) || (rc = check_out(y, y32 ? 4 : es, work, &oy)))
    return rc;
  if (!work) return SKA_OK;
  if (!gamma || !saved) return SKA_ERR_NULL;
  if (reinterpret_cast<uintptr_t>(saved) % 256) return SKA_ERR_ALIGN;
  const ska::SavedLayout L = ska::saved_layout(d.B, d.H, d.C, d.SW, d.r, d.P);
  if (saved_bytes < L.fwd) return SKA_ERR_WORKSPACE;
  // the chunk operators for the backward are kept only in a buffer of the whole size
  const bool keep_ops = saved_bytes >= L.total;
  if (y32 && !ska::fwd_tc_readout<__nv_bfloat16>(d, izq, oy)) return SKA_ERR_UNSUPPORTED;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (io_dtype == SKA_DTYPE_F32)
    e = ska::launch_fwd<float>(d, iz, izq, iv, gamma, oy, L, static_cast<char*>(saved), st, false, false);
  else
    e = ska::launch_fwd<__nv_bfloat16>(d, iz, izq, iv, gamma, oy, L, static_cast<char*>(saved), st, y32,
                                       keep_ops);
  return e == cudaSuccess ? SKA_OK : SKA_ERR_LAUNCH;
}

int ska_bwd(const SkaShape* shape, int io_dtype, const SkaTensor* z, const SkaTensor* zq, const SkaTensor* v,
            const float* gamma, const SkaTensor* dy, const void* saved, size_t saved_bytes, void* scratch,
            size_t scratch_bytes, const SkaTensor* dz, const SkaTensor* dzq, const SkaTensor* dv, float* dgamma,
            void* stream) {
  Dims d{};
  int rc = make_dims(shape, &d);
  if (rc) return rc;
  const int es = elem_size(io_dtype);
  if (!es) return SKA_ERR_DTYPE;
  const bool work = d.B > 0;
  ska::In iz{}, izq{}, iv{}, idy{};
  ska::Out odz{}, odzq{}, odv{};
  if ((rc = check_tensor(z, es, work, &iz)) || (rc = check_tensor(zq, es, work, &izq)) ||
      (rc = check_tensor(v, es, work, &iv)) || (rc = check_tensor(dy, es, work, &idy)) ||
      (rc = check_out(dz, es, work, &odz)) || (rc = check_out(dzq, es, work, &odzq)) ||
      (rc = check_out(dv, es, work, &odv)))
    return rc;
  if (!dgamma) return SKA_ERR_NULL;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (!work) {
    return cudaMemsetAsync(dgamma, 0, sizeof(float), st) == cudaSuccess ? SKA_OK : SKA_ERR_LAUNCH;
  }
  if (!gamma || !saved || !scratch) return SKA_ERR_NULL;
  if (reinterpret_cast<uintptr_t>(saved) % 256 || reinterpret_cast<uintptr_t>(scratch) % 256) return SKA_ERR_ALIGN;
  const ska::SavedLayout L = ska::saved_layout(d.B, d.H, d.C, d.SW, d.r, d.P);
  const ska::ScratchLayout S = ska::scratch_layout(d.B, d.H, d.C, d.SW, d.r, d.P);
  if (saved_bytes < L.total || scratch_bytes < S.total) return SKA_ERR_WORKSPACE;
  cudaError_t e;
  if (io_dtype == SKA_DTYPE_F32)
    e = ska::launch_bwd<float>(d, iz, izq, iv, gamma, idy, L, static_cast<const char*>(saved), S,
                               static_cast<char*>(scratch), odz, odzq, odv, dgamma, st);
  else
    e = ska::launch_bwd<__nv_bfloat16>(d, iz, izq, iv, gamma, idy, L, static_cast<const char*>(saved), S,
                                       static_cast<char*>(scratch), odz, odzq, odv, dgamma, st);
  return e == cudaSuccess ? SKA_OK : SKA_ERR_LAUNCH;
}

// ---- recurrent (decode) path ----

int ska_state_size(const SkaShape* shape, size_t* state_bytes) {
  Dims d{};
  const int rc = make_dims(shape, &d);
  if (rc) return rc;
  if (state_bytes) *state_bytes = ska::state_layout(d.B, d.H, d.r, d.P).total;
  return SKA_OK;
}

static int check_state(const Dims& d, const void* state, size_t state_bytes, ska::StateLayout* L) {
  if (!state) return SKA_ERR_NULL;
  if (reinterpret_cast<uintptr_t>(state) % 256) return SKA_ERR_ALIGN;
  *L = ska::state_layout(d.B, d.H, d.r, d.P);
  return state_bytes < L->total ? SKA_ERR_WORKSPACE : SKA_OK;
}

int ska_state_init(const SkaShape* shape, void* state, size_t state_bytes, void* stream) {
  Dims d{};
  int rc = make_dims(shape, &d);
  if (rc) return rc;
  if (d.B == 0) return SKA_OK;
  ska::StateLayout L{};
  if ((rc = check_state(d, state, state_bytes, &L))) return rc;
  return ska::launch_state_init(d, static_cast<char*>(state), L, static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? SKA_OK
             : SKA_ERR_LAUNCH;
}

int ska_prefill_state(const SkaShape* shape, int io_dtype, const SkaTensor* z, const SkaTensor* v, const void* saved,
                      size_t saved_bytes, void* state, size_t state_bytes, void* stream) {
  Dims d{};
  int rc = make_dims(shape, &d);
  if (rc) return rc;
  if (d.decay) return SKA_ERR_STRATEGY;   // the reference's state is the plain (undecayed) sum
  const int es = elem_size(io_dtype);
  if (!es) return SKA_ERR_DTYPE;
  const bool work = d.B > 0;
  ska::In iz{}, iv{};
  if ((rc = check_tensor(z, es, work, &iz)) || (rc = check_tensor(v, es, work, &iv))) return rc;
  if (!work) return SKA_OK;
  ska::StateLayout L{};
  if ((rc = check_state(d, state, state_bytes, &L))) return rc;
  if (!saved) return SKA_ERR_NULL;
  if (reinterpret_cast<uintptr_t>(saved) % 256) return SKA_ERR_ALIGN;
  const ska::SavedLayout S = ska::saved_layout(d.B, d.H, d.C, d.SW, d.r, d.P);
  if (saved_bytes < S.fwd) return SKA_ERR_WORKSPACE;
  const char* sv = static_cast<const char*>(saved);
  const float* stats = reinterpret_cast<const float*>(sv + S.stats);
  const auto* cmax = reinterpret_cast<const unsigned long long*>(sv + S.cmax);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  char* sp = static_cast<char*>(state);
  const cudaError_t e = io_dtype == SKA_DTYPE_F32
                            ? ska::launch_prefill_state<float>(d, iz, iv, stats, cmax, sp, L, st)
                            : ska::launch_prefill_state<__nv_bfloat16>(d, iz, iv, stats, cmax, sp, L, st);
  return e == cudaSuccess ? SKA_OK : SKA_ERR_LAUNCH;
}

int ska_step(const SkaShape* shape, int io_dtype, const SkaTensor* z, const SkaTensor* zq, const SkaTensor* v,
             const float* gamma, const SkaTensor* y, void* state, size_t state_bytes, void* stream) {
  Dims d{};
  int rc = make_dims(shape, &d);
  if (rc) return rc;
  if (d.decay) return SKA_ERR_STRATEGY;
  if (d.r > 32) return SKA_ERR_UNSUPPORTED;
  const int es = elem_size(io_dtype);
  if (!es) return SKA_ERR_DTYPE;
  const bool work = d.B > 0;
  ska::In iz{}, izq{}, iv{};
  ska::Out oy{};
  if ((rc = check_tensor(z, es, work, &iz)) || (rc = check_tensor(zq, es, work, &izq)) ||
      (rc = check_tensor(v, es, work, &iv)) || (rc = check_out(y, es, work, &oy)))
    return rc;
  if (!work) return SKA_OK;
  if (!gamma) return SKA_ERR_NULL;
  ska::StateLayout L{};
  if ((rc = check_state(d, state, state_bytes, &L))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  char* sp = static_cast<char*>(state);
  const cudaError_t e = io_dtype == SKA_DTYPE_F32
                            ? ska::launch_step<float>(d, iz, izq, iv, gamma, oy, sp, L, st)
                            : ska::launch_step<__nv_bfloat16>(d, iz, izq, iv, gamma, oy, sp, L, st);
  return e == cudaSuccess ? SKA_OK : SKA_ERR_LAUNCH;
}

}  // extern "C"
