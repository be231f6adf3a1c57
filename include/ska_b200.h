/*
 * ska_b200.h -- C ABI of the B200 (sm_100a) Spectral Koopman Attention core.
 *
 * The "SKA core" is the part of the reference SKAModule.forward between the
 * key/query/value projections and the eta/out_proj epilogue:
 *
 *     (z, zq, v, ssn_gamma) -> y_hat            forward
 *     (dy_hat, ...)         -> dz, dzq, dv, dgamma   backward
 *
 * Reference interface replaced (paths relative to the upstream project root,
 * KLF = koopman-lm-fast):
 *   - KLF/koopman_lm/ska.py:432-457   fp32 upcast, max-key-norm scaling, chunk
 *                                      statistics, Cholesky, post-Cholesky chain
 *   - KLF/koopman_lm/ska.py:73-151    _compute_chunk_stats_and_cholesky
 *   - KLF/koopman_lm/ska.py:158-187   _post_cholesky_pytorch
 *   - KLF/koopman_lm/ska.py:263-330   _post_cholesky_triton (+ its kernel 196-260)
 *   - KLF/koopman_lm/adaptive_chunking.py:171-256  compute_chunk_stats_decay
 *   - the PyTorch autograd backward of all of the above (the reference has no
 *     hand-written backward).
 *
 * Conventions
 *   - Every tensor is [B, T, H, D] with the last (feature) dimension
 *     contiguous; the three other strides are given in ELEMENTS and may be
 *     arbitrary (e.g. column slices of one fused projection output).
 *   - io_dtype selects the element type of z, zq, v, y, dy, dz, dzq, dv:
 *     SKA_DTYPE_F32 or SKA_DTYPE_BF16 (or, for ska_fwd, SKA_DTYPE_BF16_Y32).
 *     All arithmetic is fp32 (the reference upcasts with .float(),
 *     ska.py:436-438).
 *   - gamma / dgamma are device pointers to one fp32 scalar; dgamma is
 *     OVERWRITTEN (not accumulated).
 *   - The caller owns all memory.  ska_fwd writes a "saved" buffer that
 *     ska_bwd reads; ska_bwd also needs a scratch buffer.  Their sizes come
 *     from ska_workspace_size.  The library never allocates, never frees and
 *     never synchronises the host; work is enqueued on `stream`
 *     (a cudaStream_t, NULL = legacy default stream).
 *   - Return value: 0 on success, a negative SKA_ERR_* code otherwise (no
 *     work is enqueued on error).  A Cholesky failure is not an error: as in
 *     the reference (ska.py:140-145), a slice whose factorisation fails is
 *     refactored with 1e-4 added to the diagonal.
 */
#ifndef SKA_B200_H
#define SKA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SKA_ABI_VERSION 1

enum {
  SKA_DTYPE_F32 = 0,
  SKA_DTYPE_BF16 = 1,
  /* ska_fwd only: bf16 z, zq, v and an fp32 y (what the reference's module
   * produces under autocast: bf16 projections, fp32 core output).  Needs the
   * tensor-core readout layout (SKA_PATH_TC_READOUT_FWD) and returns
   * SKA_ERR_UNSUPPORTED otherwise.  ska_bwd of such a forward takes
   * SKA_DTYPE_BF16 (a bf16 dy). */
  SKA_DTYPE_BF16_Y32 = 2,
};

enum {
  SKA_STRATEGY_STANDARD = 0, /* ska.py:114-133                       */
  SKA_STRATEGY_DECAY = 1,    /* adaptive_chunking.py:213-238         */
};

enum {
  SKA_OK = 0,
  SKA_ERR_NULL = -1,        /* a required pointer is NULL                          */
  SKA_ERR_SHAPE = -2,       /* B<0, T<1, H<1, r<1, P<1, chunk<1, power_K<0 ...      */
  SKA_ERR_UNSUPPORTED = -3, /* r > 64, P > 128, chunk > 256, power_K > 8            */
  SKA_ERR_DTYPE = -4,       /* unknown io_dtype                                     */
  SKA_ERR_WORKSPACE = -5,   /* saved / scratch buffer too small                    */
  SKA_ERR_ALIGN = -6,       /* misaligned pointer or stride                        */
  SKA_ERR_LAUNCH = -7,      /* a kernel launch failed (cudaGetLastError)           */
  SKA_ERR_STRATEGY = -8,    /* unknown strategy, or decay_alpha not finite         */
  SKA_ERR_TIMEOUT = -9,     /* ska_check_status: a bounded wait of a tensor-core   */
                            /* kernel expired (the chunk's outputs are NaN)        */
};

/* Static problem description (constructor arguments of the reference
 * SKAModule, ska.py:368-371, plus the activation shape). */
typedef struct SkaShape {
  int64_t B;          /* batch                                              */
  int64_t T;          /* sequence length (any T >= 1; the tail is padded)   */
  int64_t H;          /* heads                                              */
  int64_t r;          /* Koopman rank (key/query dim per head), 1..64       */
  int64_t P;          /* value dim per head, 1..128                         */
  int64_t chunk_size; /* CS, 1..256                                         */
  int32_t power_K;    /* filter power, 0..8                                 */
  int32_t strategy;   /* SKA_STRATEGY_*                                     */
  float ridge_eps;    /* ridge added to the Gram diagonal                   */
  float decay_alpha;  /* decay strategy only                                */
} SkaShape;

/* One [B, T, H, D] tensor: data pointer + element strides (feature stride 1). */
typedef struct SkaTensor {
  void* data;
  int64_t stride_b;
  int64_t stride_t;
  int64_t stride_h;
} SkaTensor;

/* ABI version (SKA_ABI_VERSION of the built library). */
int ska_abi_version(void);

/* Static string for a return code. */
const char* ska_status_string(int code);

/* Bytes needed for the forward's saved buffer (read by ska_bwd) and for the
 * backward's scratch buffer.  Either output pointer may be NULL. */
int ska_workspace_size(const SkaShape* shape, size_t* saved_bytes, size_t* scratch_bytes);

/* Bytes of the saved buffer for a forward that no ska_bwd will follow
 * (inference, prefill; no counterpart in the reference, whose autograd keeps
 * what it keeps).  It is the leading part of ska_workspace_size's saved_bytes:
 * statistics, norms and the readout operands, without the chunk operators
 * (Li, A, A^K, U, V, S) that the bf16 backward reads.  ska_fwd given at least
 * this but fewer than saved_bytes does not write those operators; ska_bwd
 * checks saved_bytes >= ska_workspace_size's and must be given the buffer of a
 * forward that was given that many. */
int ska_forward_workspace_size(const SkaShape* shape, size_t* saved_bytes);

/* Forward.  Replaces ska.py:436-457 between the projections and eta:
 *   y = SKA_core(z, zq, v; ssn_gamma)   (y in io_dtype, [B,T,H,P]).
 * `saved` must hold ska_workspace_size(...).saved_bytes when ska_bwd will
 * follow (its contents are consumed by ska_bwd for the same inputs), else at
 * least ska_forward_workspace_size(...) bytes. */
int ska_fwd(const SkaShape* shape, int io_dtype,
            const SkaTensor* z, const SkaTensor* zq, const SkaTensor* v,
            const float* gamma, const SkaTensor* y,
            void* saved, size_t saved_bytes, void* stream);

/* Backward of ska_fwd (what PyTorch autograd computes for the reference's
 * PyTorch backend): given dy, writes dz, dzq, dv (io_dtype) and *dgamma (fp32,
 * overwritten).  z, zq, v, gamma and `saved` must be those of the forward. */
int ska_bwd(const SkaShape* shape, int io_dtype,
            const SkaTensor* z, const SkaTensor* zq, const SkaTensor* v,
            const float* gamma, const SkaTensor* dy,
            const void* saved, size_t saved_bytes,
            void* scratch, size_t scratch_bytes,
            const SkaTensor* dz, const SkaTensor* dzq, const SkaTensor* dv,
            float* dgamma, void* stream);

/* Profiling hook (process-wide, not thread-safe; no counterpart in the
 * reference, which has no per-kernel timing).  With `events` non-NULL and
 * count >= SKA_PROFILE_EVENTS, every later ska_fwd records events[0] on its
 * stream before its first kernel, events[1..3] after the statistics, the scan
 * and the chunk-operator kernels, and events[9] after the tensor-core readout
 * kernel; ska_bwd records events[4] before its first kernel and events[5..8]
 * after the readout-gradient kernel, the chunk operators, the scan and the
 * token kernel.  An event whose kernel does not run for the layout is recorded
 * right after the previous one.  The handles are cudaEvent_t values created
 * by the caller.  NULL disables recording. */
#define SKA_PROFILE_EVENTS 10
int ska_set_profile_events(void* const* events, int count);

/* Which kernels ska_fwd / ska_bwd launch for these arguments (no counterpart in
 * the reference; for integrators checking that a layout reaches the fast
 * kernels).  Returns a non-negative mask of SKA_PATH_* bits, or a negative
 * SKA_ERR_* code for arguments ska_fwd would reject.  Launches nothing.
 *   SKA_PATH_TC_STATS    chunk statistics on TMA + tcgen05 (bf16 tensors with
 *                        16-byte aligned base and strides, r % 16 == 0,
 *                        P % 8 == 0, chunk_size % 16 == 0); otherwise on
 *                        CUDA-core fp32 kernels
 *   SKA_PATH_WARP_CHUNK  chunk operators on the warp-per-chunk register
 *                        kernels (r <= 32); otherwise one CTA per chunk
 *   SKA_PATH_TC_TOKEN_BWD  per-token dz, dv on TMA + tcgen05 (as TC_STATS, plus
 *                        chunk_size <= 128 and P % 16 == 0, with dz and dv laid
 *                        out like z and v); otherwise on CUDA cores
 *   SKA_PATH_TC_READOUT_BWD  the readout gradient (dW and dzq) on TMA + tcgen05
 *                        too, and the chunk operators' backward without a token
 *                        pass (TC_TOKEN_BWD and WARP_CHUNK, with zq, dy and dzq
 *                        laid out like z and v); otherwise inside the chunk
 *                        kernel
 *   SKA_PATH_FUSED_SCAN  the forward statistics and their prefix scan in one
 *                        kernel, one CTA per (batch, head) series (TC_STATS,
 *                        r = 32, P <= 64 and B * H >= 64); otherwise two
 *   SKA_PATH_TC_READOUT_FWD  the forward readout y = (W / m) zq as its own TMA +
 *                        tcgen05 kernel (bf16, WARP_CHUNK or QUAD_CHUNK, r % 16 == 0,
 *                        P % 16 == 0, chunk_size <= 128, y laid out like v);
 *                        otherwise inside the chunk-operator kernel
 *   SKA_PATH_QUAD_CHUNK  forward chunk operators for 32 < r <= 64 (r % 8 == 0,
 *                        P <= 64, bf16 with a TC_READOUT_FWD layout) on the
 *                        four-warp kernel (one CTA per chunk, blocked
 *                        Cholesky); otherwise, for r > 32, on the one-CTA
 *                        CUDA-core kernel
 *   SKA_PATH_TC_CHUNK_FWD  forward chunk operators for r <= 32 on tcgen05, four
 *                        chunks per CTA with their r x r products batched into
 *                        one 128 x 128 product (bf16, WARP_CHUNK and
 *                        TC_READOUT_FWD); otherwise on the warp-per-chunk kernel
 *   SKA_PATH_TC_CHUNK_BWD  the backward's chunk operators the same way (bf16,
 *                        TC_READOUT_BWD, r % 16 == 0, power_K <= 2); otherwise
 *                        warp per chunk
 *   SKA_PATH_QUAD_CHUNK_BWD  the backward's chunk operators for 32 < r <= 64 on
 *                        four warps per chunk from the operators the forward
 *                        kept (QUAD_CHUNK shapes with TC_READOUT_BWD and
 *                        power_K <= 2); otherwise one CTA per chunk that
 *                        recomputes the forward */
#define SKA_PATH_TC_STATS 1
#define SKA_PATH_WARP_CHUNK 2
#define SKA_PATH_TC_TOKEN_BWD 4
#define SKA_PATH_TC_READOUT_BWD 8
#define SKA_PATH_FUSED_SCAN 16
#define SKA_PATH_TC_READOUT_FWD 32
#define SKA_PATH_QUAD_CHUNK 64
#define SKA_PATH_TC_CHUNK_FWD 128
#define SKA_PATH_TC_CHUNK_BWD 256
#define SKA_PATH_QUAD_CHUNK_BWD 512
int ska_kernel_path(const SkaShape* shape, int io_dtype, const SkaTensor* z, const SkaTensor* v);

/* Bounded waits of the tensor-core kernels (no counterpart in the reference,
 * whose library calls have no device-side waits; this is the "scan-wait
 * timeout" error of the drop-in contract).  Every mbarrier wait in the TMA +
 * tcgen05 kernels gives up after a bounded number of polls.  A wait that gives
 * up records a status entry for its chunk, waits (with the full limit) for the
 * copies and products still in flight, writes NaN into that chunk's outputs,
 * frees its tensor memory and returns: the launch completes and the CUDA
 * context stays usable.  ska_fwd / ska_bwd cannot report this at return (they
 * never synchronise); ska_check_status reads it afterwards.
 *
 * Status entries: int32 [B][H][C] (chunk c of head h of batch b at
 * (b * H + h) * C + c), one array in `saved` (forward: bits 0-1 the statistics
 * kernel, bits 2-3 the readout kernel, bits 4-5 the tensor-core chunk-operator
 * kernel; each 0 ok, 1 copy wait expired, 2 product wait expired) and one in `scratch` (backward: bits 0-1 the
 * readout-gradient kernel, bits 2-3 the token kernel, bits 4-5 the tensor-core
 * chunk-operator kernel, coded the same way).
 * Layouts without tensor-core kernels write 0.
 *
 * ska_check_status synchronises `stream`, then scans the forward entries of
 * `saved` and the backward entries of `scratch` (either may be NULL to skip it).
 * Returns SKA_OK when every entry is 0, SKA_ERR_TIMEOUT at the first non-zero one
 * with *first_bad = its flat chunk index and *code = the forward entry's bits or
 * SKA_STATUS_BWD_BASE + the backward entry's bits; other negative codes for bad
 * arguments.  A diagnostic call: it copies the entries to host memory.
 *
 * ska_set_wait_limit sets the poll limit of the first wait of every role in
 * every later launch (process-wide; 0 = give up at once, without polling;
 * 0xFFFFFFFF = back to the default of 2^22 polls).  The waits that drain
 * in-flight work after a failure always keep the default.  It exists so that a
 * test can make the waits expire on a GPU without a fault. */
#define SKA_STATUS_BWD_BASE 16
int ska_set_wait_limit(uint32_t polls);
int ska_check_status(const SkaShape* shape, const void* saved, size_t saved_bytes, const void* scratch,
                     size_t scratch_bytes, void* stream, int64_t* first_bad, int* code);

/* ---- Recurrent (decode) path --------------------------------------------
 * Replaces KLF/koopman_lm/recurrent.py for one SKA layer: SKAState (:48-66),
 * the state extraction of _ska_prefill (:129-189) and _ska_step (:270-375).
 * The state of one layer is one caller-owned buffer of ska_state_size bytes
 * (256-byte aligned), fp32 arrays in this order, each 256-byte aligned:
 *   G [B][H][r][r], M [B][H][r][r], C_v [B][H][P][r], z_last [B][H][r],
 *   max_norm [B][H], flags [B][H] (int32, bit 0: z_last is set).
 * G, M and C_v hold the statistics of the keys normalised by max_norm, G with the
 * ridge on its diagonal, exactly as the reference's SKAState.  Only B, H, r, P
 * (and for the calls below T, ridge_eps, power_K, chunk_size) of the shape are
 * used; the standard strategy only (the reference's state is the undecayed sum):
 * SKA_STRATEGY_DECAY returns SKA_ERR_STRATEGY. */
int ska_state_size(const SkaShape* shape, size_t* state_bytes);

/* The fresh state of SKAState.__init__: G = ridge I, M = C_v = 0, no z_last,
 * max_norm = 1e-6. */
int ska_state_init(const SkaShape* shape, void* state, size_t state_bytes, void* stream);

/* The state after a prompt of shape->T tokens (recurrent.py:150-189), from the
 * `saved` buffer that ska_fwd wrote for the same shape, z and v: the exclusive
 * prefix statistics of the last chunk plus that chunk's own tokens (the rest of
 * the prompt is not read again), scaled by the forward's max key norm, which
 * becomes the state's max_norm; z_last = z[T-1] / max_norm.  saved_bytes >=
 * ska_forward_workspace_size(...). */
int ska_prefill_state(const SkaShape* shape, int io_dtype, const SkaTensor* z, const SkaTensor* v,
                      const void* saved, size_t saved_bytes, void* state, size_t state_bytes, void* stream);

/* shape->T decode tokens in order (z, zq, v: [B, T, H, D]; y: [B, T, H, P]),
 * each exactly one _ska_step (recurrent.py:306-369): with max_norm frozen,
 * G += z z^T, M += z z_last^T (when z_last is set), C_v += v z^T, then
 * y = C_v G^-1 L A^K L^-1 zq with L = chol(sym(G)) (1e-4 jitter where that
 * fails) and A = clamp(gamma,1,1.5) (M G^-1) / max(sigma, 1) from 6 power
 * iterations.  Updates the state in place.  r <= 32 (SKA_ERR_UNSUPPORTED
 * otherwise).  One warp per (batch, head). */
int ska_step(const SkaShape* shape, int io_dtype, const SkaTensor* z, const SkaTensor* zq, const SkaTensor* v,
             const float* gamma, const SkaTensor* y, void* state, size_t state_bytes, void* stream);

/* Forward with no allocation anywhere (no counterpart in the reference, whose
 * PyTorch path always allocates through the caching allocator).  Same
 * computation and arguments as ska_fwd, minus the `saved` buffer: the
 * workspace is a fixed array of SKA_NOALLOC_SCRATCH_BYTES compiled into this
 * library as device memory, which every GPU that loads the library holds until
 * the process exits.  It serves callers that cannot call cudaMalloc: FFI hosts
 * with no CUDA allocator of their own, and inference loops that must not
 * allocate between launches (cudaMalloc can synchronise the device).
 *   - Problems whose ska_forward_workspace_size exceeds
 *     SKA_NOALLOC_SCRATCH_BYTES return SKA_ERR_WORKSPACE and launch nothing.
 *     The checks run in this order: the shape (as ska_workspace_size), then
 *     the size against the array, then everything ska_fwd checks (dtype,
 *     pointers, alignment); so an over-size problem returns SKA_ERR_WORKSPACE
 *     whatever its tensors are.
 *   - The first call on each device looks up the array's device address
 *     (cudaGetSymbolAddress) with that device current; make that first call
 *     before any stream capture.  The address is kept for the life of the
 *     process, so a device reset (cudaDeviceReset, or destroying the primary
 *     context) is not supported once the entry point has been called.
 *   - All calls share the one array and it keeps the previous call's contents
 *     (every part of it that is read is rewritten first).  Calls whose work
 *     overlaps on the GPU race on it: serialise them, e.g. on one stream.
 *   - Forward only: ska_bwd still needs the `saved` buffer of ska_fwd. */
#define SKA_NOALLOC_SCRATCH_BYTES (16u << 20)
int ska_fwd_noalloc(const SkaShape* shape, int io_dtype,
                    const SkaTensor* z, const SkaTensor* zq, const SkaTensor* v,
                    const float* gamma, const SkaTensor* y, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SKA_B200_H */
