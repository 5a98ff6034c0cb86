/*
 * pathtile_b200.h -- C ABI of the B200 (sm_100a) short depthwise Conv1D
 * training path: forward (FWD), input gradient (dX) and weight gradient (dK),
 * FP32, for sequence length L <= 48 and filter length K <= 48.
 *
 * Layout: activations are contiguous float32 [B, H, L] (one contiguous row of
 * L floats per (batch b, channel h) sequence); filters and filter gradients
 * are contiguous float32 [H, K].  All pointers are DEVICE pointers of the
 * calling thread's current CUDA device and must be 16-byte aligned (every
 * cudaMalloc / PyTorch allocation is).  `stream` is a cudaStream_t (NULL is
 * the legacy default stream).  Every call is asynchronous with respect to the
 * host; errors found before launch are reported synchronously.
 *
 * Padding convention ("same" output length, as the reference PyTorch path
 * F.pad(x, (K//2, K-1-K//2)) + grouped conv1d,
 * benchmark/benchmark_shape_sweep_ampere.py:220-239):
 *   y [b,h,t] = sum_{j<K} x [b,h,t+j-K/2] * k[h,j]         (zero outside 0..L-1)
 *   dx[b,h,t] = sum_{j<K} dy[b,h,t-j+K/2] * k[h,j]
 *   dk[h,j]   = sum_{b,t} dy[b,h,t] * x[b,h,t+j-K/2]
 *
 * Status codes follow the external-kernel bridge convention of the reference
 * (benchmark/flashdwc_fp32_bridge.cu:15-20: 0 = ok, -2 = bad arguments);
 * the other negative values are specific to this library.
 */
#ifndef PATHTILE_B200_H_
#define PATHTILE_B200_H_

#include <stddef.h>

#if defined(__GNUC__)
#define PT_API __attribute__((visibility("default")))
#else
#define PT_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define PT_OK 0
#define PT_ERR_ARGS (-2)        /* null pointer, non-positive or mismatched dims */
#define PT_ERR_UNSUPPORTED (-3) /* L > 48 or K > 48 (kernels are specialised) */
#define PT_ERR_ALIGN (-4)       /* a pointer is not 16-byte aligned */
#define PT_ERR_WORKSPACE (-5)   /* deterministic dK workspace missing or too small */
#define PT_ERR_CUDA (-6)        /* a CUDA runtime/driver call or launch failed */
#define PT_ERR_DEVICE (-7)      /* current device is not compute capability 10.x */
#define PT_ERR_SCRATCH_LIMIT (-8) /* pt_dk_noalloc: shape needs more than its fixed scratch */

#define PT_MAX_L 48
#define PT_MAX_K 48

/* dK reduction modes (pt_dk `mode`). */
#define PT_DK_ATOMIC 0          /* one float atomicAdd per (CTA, h, j): dk += dK (dk pre-zeroed by caller) */
#define PT_DK_DETERMINISTIC 1   /* two passes through a [CTA][K][h] workspace: dk = dK, bit-reproducible */
#define PT_DK_DETERMINISTIC_ACCUMULATE 2 /* as 1, but dk += dK */

/* Paths for pt_config / pt_set_config. */
#define PT_PATH_FWD 0
#define PT_PATH_DX 1
#define PT_PATH_DK 2
#define PT_PATH_BWD_FUSED 3  /* pt_kernel_info only: the fused dX + dK kernel of pt_dx_dk */

/* Engines (pt_set_engine, pt_config out[6]). */
#define PT_ENGINE_FFMA 0    /* CUDA-core FP32 FMA kernels: every path and shape */
#define PT_ENGINE_TENSOR 1  /* tcgen05 tensor cores, FP32-accurate 3xTF32 split, L % 4 == 0 */

/*
 * Forward pass.  Replaces the reference launch of dwconv1d_warptile_fwd via
 * AmpereWarpRuntime.launch_fwd (kernels/warp_tiled_ampere.py:723-747, kernel
 * :372-434) and, behind the legacy name surface, dwconv1d_fwd_shared
 * (kernels/warp_tiled.py:151, launched at :853-885).
 */
PT_API int pt_fwd(const float* x, const float* k, float* y, int B, int H, int L, int K,
           void* stream);

/*
 * Input gradient.  Replaces AmpereWarpRuntime.launch_bwd_input
 * (kernels/warp_tiled_ampere.py:749-773, kernel :440-502) and
 * dwconv1d_bwd_input_shared (kernels/warp_tiled.py:297, launched at :926-963).
 */
PT_API int pt_dx(const float* dy, const float* k, float* dx, int B, int H, int L, int K,
          void* stream);

/*
 * Weight gradient.  Replaces AmpereWarpRuntime.launch_bwd_weight
 * (kernels/warp_tiled_ampere.py:775-812, kernel :509-619; atomic semantics:
 * dk must be zeroed by the caller, :890-893) and the deterministic two-pass
 * path dwconv1d_warptile_bwd_weight_partials + dwconv1d_warptile_reduce_partials
 * (kernels/warp_tiled_noatomic_optimized.py:881-1150, launched at :1473-1550).
 * `ws`/`ws_bytes` is the caller-owned workspace of the deterministic modes
 * (ignored by PT_DK_ATOMIC); its size is pt_dk_workspace_bytes(B,H,L,K).
 */
PT_API int pt_dk(const float* dy, const float* x, float* dk, int B, int H, int L, int K,
          int mode, void* ws, size_t ws_bytes, void* stream);

/*
 * Deterministic weight gradient that allocates nothing; it has no counterpart
 * in the reference.  For callers that may not allocate device memory (a
 * runtime that owns a fixed memory budget and every allocation in it, or a
 * steady-state loop where cudaMalloc/cudaFree would block on the device): the
 * per-CTA partial sums go to a fixed scratch array inside the library
 * (PT_DK_NOALLOC_SCRATCH_BYTES = 8 MiB of device memory, held by every GPU
 * that loads the library until the process exits) instead of a caller
 * workspace.  dk = dK, or dk += dK when `accumulate` is non-zero; results are
 * identical to pt_dk in PT_DK_DETERMINISTIC mode.  Returns
 * PT_ERR_SCRATCH_LIMIT when pt_dk_workspace_bytes(B,H,L,K) exceeds the
 * scratch size (the primary B=16384,H=128,L=K=48 shape needs 7.3 MB).  The
 * first call on each device resolves the array's device address and must be
 * made before any stream capture; calls that overlap on the GPU share the one
 * array and race, so the caller serialises them.
 */
#define PT_DK_NOALLOC_SCRATCH_BYTES (8u * 1024u * 1024u)
PT_API int pt_dk_noalloc(const float* dy, const float* x, float* dk, int B, int H, int L, int K,
                         int accumulate, void* stream);

/*
 * Input and filter gradients in one call: dx as pt_dx, dk as pt_dk (same
 * modes and workspace rules; query pt_dx_dk_workspace_bytes).  One kernel
 * reads dy and x once and writes dx wherever a fused kernel applies:
 *  - the tensor-core one (dX on tcgen05, dK on the CUDA cores) for rows of
 *    32 < L <= 48 columns with L % 4 == 0 and any K <= 48, unless dX is forced
 *    onto the CUDA cores, where the grid can give every CTA a single channel
 *    (no workspace when each channel has one CTA);
 *  - otherwise the CUDA-core one for every (L, K) with a specialised CUDA-core
 *    kernel (and H*L % 4 == 0 when L % 4 != 0), unless dX or dK is forced onto
 *    the tensor cores;
 * other shapes run pt_dx then pt_dk.  The reference launches the two
 * separately (DepthConvAmpere.backward, kernels/warp_tiled_ampere.py:882-898);
 * no fused counterpart.
 */
PT_API int pt_dx_dk(const float* dy, const float* x, const float* k, float* dx, float* dk, int B, int H,
                    int L, int K, int mode, void* ws, size_t ws_bytes, void* stream);

/*
 * Channels-last variants: x, y, dy, dx are [B, L, H] (H contiguous), k and dk
 * [H, K], same math as pt_fwd / pt_dx / pt_dk.  They replace the S4 block's
 * transposes to [B, H, L] and back around the convolution
 * (kernels/warp_tiled_ampere.py:1186, :1190).  CUDA-core kernels, one thread
 * per (b, h) sequence; pointers need 4-byte alignment (ws: 16).  pt_dk_cl is
 * deterministic (per-CTA partials in ws, then a fixed-order sum): dk = dK, or
 * dk += dK when accumulate != 0.
 */
PT_API int pt_fwd_cl(const float* x, const float* k, float* y, int B, int L, int H, int K, void* stream);
PT_API int pt_dx_cl(const float* dy, const float* k, float* dx, int B, int L, int H, int K, void* stream);
PT_API int pt_dk_cl(const float* dy, const float* x, float* dk, int B, int L, int H, int K, int accumulate,
                    void* ws, size_t ws_bytes, void* stream);
/* Workspace bytes pt_dk_cl needs for this shape on the current device (0 if invalid). */
PT_API size_t pt_dk_cl_workspace_bytes(int B, int L, int H, int K);

/* Kernel pt_dx_dk runs for this shape on the current device: 1 the tensor-core
 * fused kernel, 2 the CUDA-core fused kernel, 0 pt_dx then pt_dk. */
PT_API int pt_dx_dk_fused(int B, int H, int L, int K);

/* Workspace bytes pt_dx_dk needs for this shape (0 for invalid shapes or none needed). */
PT_API size_t pt_dx_dk_workspace_bytes(int B, int H, int L, int K);

/*
 * Bytes of deterministic-dK workspace for this shape under the active launch
 * configuration on the current device (the reference sizes its cached
 * [H,K,num_btiles] buffer at kernels/warp_tiled_noatomic_optimized.py:1448-1471).
 * Returns 0 for invalid shapes.
 */
PT_API size_t pt_dk_workspace_bytes(int B, int H, int L, int K);

/*
 * Launch configuration that the frozen PathTile table selects for `path`
 * (PT_PATH_*) at this shape.  out[0] = rows per tile, out[1] = pipeline
 * stages, out[2] = CTAs per SM, out[3] = 1 if an (L,K)-specialised kernel
 * exists, else 0 (generic kernel); if `n` >= 5, out[4] = the shape's
 * arithmetic-intensity class keying the table (0 light, 1 medium, 2 heavy:
 * in-range FMAs per output element < 12, < 24, else); if `n` >= 6, out[5] =
 * consumer threads per row (1, or 2 when two threads split a row); if `n` >= 7,
 * out[6] = the engine that runs (PT_ENGINE_*); if `n` >= 9, out[7] = the
 * backward kernel pt_dx_dk may use (PT_BWD_*) and out[8] = the most channels
 * a helper CTA of the tensor-core fused kernel may own, for the shape's class.
 * `n` >= 4.
 * Mirrors the frozen constants that the reference bakes into CUDA_TEMPLATE
 * (WARPS_PER_BLOCK / BWDK_BLOCK, kernels/warp_tiled_ampere.py:668-672,
 * selected by scripts/aggregate_pathtile_results.py:222-240).
 */
PT_API int pt_config(int path, int B, int H, int L, int K, int* out, int n);

/*
 * Override the launch configuration of `path` for all shapes (rows_per_tile in
 * {32,64,128,256}, stages in {2,3,4}, ctas_per_sm in {1,2,3,4}, threads_per_row
 * in {1,2}); passing rows_per_tile = 0 restores the frozen table.  Used by the offline PathTile
 * candidate sweep, the counterpart of recompiling CUDA_TEMPLATE per candidate
 * (benchmark/benchmark_pathtile_candidate_sweep.py:493-560).  Not thread-safe
 * with concurrent launches.
 */
PT_API int pt_set_config(int path, int rows_per_tile, int stages, int ctas_per_sm,
                         int threads_per_row);

/*
 * Engine of `path` for all shapes: PT_ENGINE_FFMA, PT_ENGINE_TENSOR, or -1 to
 * restore the frozen table.  PT_ENGINE_TENSOR applies at L % 4 == 0 only (and,
 * for dK, where every CTA's channel groups stay resident: the grid has a
 * multiple of half the group count CTAs); other shapes keep the FFMA kernels.
 * No reference counterpart (the reference has CUDA-core kernels only).  Not
 * thread-safe with concurrent launches.
 */
PT_API int pt_set_engine(int path, int engine);

/*
 * Per-call launch options, for callers that must not change the process-wide
 * choice (two runtimes in one process, a tuner beside a training job).  One
 * entry per path, indexed by PT_PATH_FWD / PT_PATH_DX / PT_PATH_DK:
 * rows_per_tile 0 takes the frozen PathTile table for that path (the other
 * three fields are then ignored), else the same ranges as pt_set_config;
 * engine -1 takes the frozen engine, else PT_ENGINE_*; bwd_kernel and
 * helper_channels select pt_dx_dk's kernel and the tensor-core fused kernel's
 * schedule (-1: frozen).  The *_ex entry points
 * below behave exactly like their plain counterparts, with `opts` in place of
 * the process-wide overrides for the duration of the call (NULL: the
 * process-wide state).  Invalid options give PT_ERR_ARGS (0 for the size
 * queries).  The reference's counterpart is one runtime compiled per
 * configuration (AmpereWarpRuntime(warps_per_block, bwdk_block),
 * kernels/warp_tiled_ampere.py:636-691).
 */
typedef struct pt_launch_opts {
  int rows_per_tile[3];
  int stages[3];
  int ctas_per_sm[3];
  int threads_per_row[3];
  int engine[3];
  int bwd_kernel;       /* pt_dx_dk: PT_BWD_* (PT_BWD_FROZEN: the frozen per-class choice) */
  int helper_channels;  /* tensor-core fused kernel: most channels one helper CTA may own
                           (0: no helper CTAs; -1: the frozen per-class limit) */
} pt_launch_opts;

/* Backward kernels pt_dx_dk may run (pt_launch_opts.bwd_kernel). */
#define PT_BWD_FROZEN (-1)        /* the frozen per-class choice */
#define PT_BWD_SEPARATE 0         /* pt_dx then pt_dk */
#define PT_BWD_TENSOR_FUSED 1     /* the tensor-core fused kernel where it applies, else separate */
#define PT_BWD_FFMA_FUSED 2       /* the CUDA-core fused kernel where it applies, else separate */
#define PT_BWD_ANY_FUSED 3        /* tensor-core fused, else CUDA-core fused, else separate */

PT_API int pt_fwd_ex(const float* x, const float* k, float* y, int B, int H, int L, int K,
                     const pt_launch_opts* opts, void* stream);
PT_API int pt_dx_ex(const float* dy, const float* k, float* dx, int B, int H, int L, int K,
                    const pt_launch_opts* opts, void* stream);
PT_API int pt_dk_ex(const float* dy, const float* x, float* dk, int B, int H, int L, int K, int mode,
                    void* ws, size_t ws_bytes, const pt_launch_opts* opts, void* stream);
PT_API int pt_dx_dk_ex(const float* dy, const float* x, const float* k, float* dx, float* dk, int B, int H,
                       int L, int K, int mode, void* ws, size_t ws_bytes, const pt_launch_opts* opts,
                       void* stream);
PT_API size_t pt_dk_workspace_bytes_ex(int B, int H, int L, int K, const pt_launch_opts* opts);
PT_API size_t pt_dx_dk_workspace_bytes_ex(int B, int H, int L, int K, const pt_launch_opts* opts);
PT_API int pt_dx_dk_fused_ex(int B, int H, int L, int K, const pt_launch_opts* opts);
PT_API int pt_config_ex(int path, int B, int H, int L, int K, int* out, int n, const pt_launch_opts* opts);
PT_API int pt_kernel_info_ex(int path, int B, int H, int L, int K, int* out, int n,
                             const pt_launch_opts* opts);

/*
 * Resources of the kernel `path` would launch for this shape: out[0] registers
 * per thread, out[1] static shared bytes, out[2] local (spill) bytes per
 * thread, out[3] threads per CTA, out[4] dynamic shared bytes, out[5] resident
 * CTAs per SM (occupancy API), out[6] grid size, out[7] 1 if specialised.
 * `n` >= 8.  `path` PT_PATH_BWD_FUSED reports the fused backward kernel of
 * pt_dx_dk (PT_ERR_UNSUPPORTED where pt_dx_dk_fused is 0).  Counterpart of AmpereWarpRuntime.resource_report, which reads the
 * compiled function's num_regs / shared_size_bytes / local_size_bytes
 * (kernels/warp_tiled_ampere.py:814-833).
 */
PT_API int pt_kernel_info(int path, int B, int H, int L, int K, int* out, int n);

/*
 * Device-side error word: kernels never spin without bound; a wait that runs
 * past its limit (2 s) sets a bit here and the kernel returns early: bit 0 a
 * consumer waited for a tile, bit 1 the producer waited for an in-flight copy
 * to drain, bit 2 the producer waited for consumers to finish a stage; the
 * tensor-core kernels add bit 3 (converter waits), bit 4 (MMA issuer waits) and
 * bit 5 (epilogue waits); bit 6 a peer's dK row never arrived (pt_dx_dk_allreduce).  Reads (and
 * with clear != 0, resets) the word of the current device; synchronises the
 * device.  The reference has no device-side error channel (its kernels return
 * silently on L > 48, kernels/warp_tiled_ampere.py:390).
 */
PT_API int pt_device_error(unsigned int* out, int clear);

/*
 * Data-parallel step on the GPUs of one node: each rank has dK of its batch
 * shard; these entry points sum dK over the ranks through the other GPUs'
 * memory (NVLink / NVSwitch), the counterpart of the step's NCCL all-reduce
 * (the reference is single-GPU; no counterpart there).  Each rank owns an
 * exchange buffer of pt_peer_buffer_bytes(world, H, K) (pt_peer_alloc: device
 * memory, zeroed) and maps every other rank's (pt_ipc_export on the owner,
 * pt_ipc_import on the others, the 64-byte handles exchanged by the caller,
 * e.g. torch.distributed).  pt_peer_group lists the buffers as mapped in this
 * process (bufs[rank] = the own one) and an epoch that the caller increases by
 * one for every call, identically on all ranks, starting at 1.  Every rank must
 * make the same calls in the same order; a rank whose peers do not arrive within
 * 2 s sets bit 6 (value 64) of the device error word and leaves dk unsummed.
 *
 * pt_dx_dk_allreduce: pt_dx_dk (deterministic: dk = dK) with dk summed over the
 * ranks; where the tensor-core fused kernel runs with one CTA per channel
 * (pt_dx_dk_allreduce_fused = 1), the CTA that computed a channel's row sends
 * it to every rank and sums the ranks' rows in its epilogue -- no separate
 * collective; otherwise pt_dx_dk then pt_allreduce_peer.  pt_allreduce_peer:
 * dk[H][K] summed over the ranks in place.  Sums run in rank order on every
 * rank, so all ranks hold the same bits.
 */
#define PT_MAX_PEERS 8
#define PT_IPC_HANDLE_BYTES 64
typedef struct pt_peer_group {
  int rank;
  int world;
  void* bufs[PT_MAX_PEERS];
  unsigned int epoch;
} pt_peer_group;

PT_API size_t pt_peer_buffer_bytes(int world, int H, int K);
PT_API int pt_peer_alloc(size_t bytes, void** ptr);
PT_API int pt_peer_free(void* ptr);
PT_API int pt_ipc_export(const void* ptr, void* handle);
PT_API int pt_ipc_import(const void* handle, void** ptr);
PT_API int pt_ipc_close(void* ptr);
PT_API int pt_dx_dk_allreduce(const float* dy, const float* x, const float* k, float* dx, float* dk, int B, int H,
                              int L, int K, void* ws, size_t ws_bytes, const pt_peer_group* grp, void* stream);
PT_API int pt_dx_dk_allreduce_fused(int B, int H, int L, int K);
PT_API int pt_allreduce_peer(float* dk, int H, int K, const pt_peer_group* grp, void* stream);

/*
 * Self-test of the device-side wait limit (test use): launches one warp that
 * waits on an mbarrier nothing ever arrives on, through the same bounded-wait
 * routine as every pipeline kernel, but limited to `limit_ns` (1 ns .. 1 s)
 * instead of 2 s.  The wait runs out, bit 0 of the device error word is set
 * (as when a consumer's tile never arrives) and the kernel returns; nothing
 * is left in flight and the context stays usable.  `out` is a 16-byte
 * aligned device buffer of two unsigned 64-bit words: the wait's duration in
 * ns and 1 if it reported success (0 expected).  No reference counterpart.
 */
PT_API int pt_selftest_wait_timeout(unsigned long long limit_ns, void* out, void* stream);

/* Human-readable text for a status code. */
PT_API const char* pt_status_string(int status);

/* CUDA error code of the last PT_ERR_CUDA on this host thread (0 if none). */
PT_API int pt_last_cuda_error(void);

/* Library version: major*10000 + minor*100 + patch. */
PT_API int pt_version(void);

#ifdef __cplusplus
}
#endif

#endif /* PATHTILE_B200_H_ */
