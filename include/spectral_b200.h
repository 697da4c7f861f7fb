/*
 * spectral_b200.h: the C ABI of the B200-native batched FFT library (libspectral_b200.so).
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream (cudaStream_t passed
 * as void*; NULL is the legacy default stream), runs on the calling thread's current device,
 * and returns a status code. On failure spectral_last_error() returns the message for the
 * calling thread. Kernels are enqueued on `stream` and return without synchronizing.
 *
 * Conventions are numpy's and torch's (norm="backward"): forward transforms are unnormalized,
 * inverse ones divide by the number of points. Transforms of a batch are stored back to back.
 * Complex values are two packed floats (re, im): complex64 / c10::complex<float> / the
 * reference's cf32 (csrc/common/types.hpp:7-12).
 *
 * `impl` names one of the registry's implementations (spectral_impl_name). The registry keeps
 * the reference's five names, order and size limits (csrc/fft/registry.hpp:28-40): "naive",
 * "stockham_r2", "stockham_r4", "stockham_r8", "stockham_r8_table".
 *
 * Workspaces: the 2D, pruned and (for "naive") real entry points take a caller-allocated `work`
 * buffer whose size in complex values the matching *_workspace function reports (0 means NULL
 * is accepted), as the reference's fft2d.hpp:27-36 and pruned.hpp:26-36 do.
 *
 * Tables: the first call on a device that needs a given twiddle table (or, for the tensor-core
 * pruned transforms, a DFT operand table) builds it in the library's static device pool with a
 * synchronous copy, as the reference's twiddle_table() does (csrc/fft/twiddles.cu:17-46); make
 * that first call before any CUDA graph capture on the device.
 */
#ifndef SPECTRAL_B200_H
#define SPECTRAL_B200_H

#include <stddef.h>

#if defined(__GNUC__)
#define SPECTRAL_API __attribute__((visibility("default")))
#else
#define SPECTRAL_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. INVALID_ARGUMENT is what the reference signals with std::invalid_argument
 * (Python ValueError); CUDA_ERROR what its CUDA_CHECK signals with std::runtime_error. */
#define SPECTRAL_OK 0
#define SPECTRAL_INVALID_ARGUMENT 1
#define SPECTRAL_CUDA_ERROR 2
#define SPECTRAL_INTERNAL_ERROR 3

/* Column methods of the 2D transforms (reference: csrc/fft/fft2d.hpp:24, enum Columns). */
#define SPECTRAL_COLUMNS_TRANSPOSE 0
#define SPECTRAL_COLUMNS_STRIDED 1

/* The message of the calling thread's last failed call ("" if none). */
SPECTRAL_API const char* spectral_last_error(void);

/* Fault codes that kernels recorded on the current device since the last clear (0: none), read
 * with a synchronizing copy; clear != 0 resets them. A kernel whose bounded wait on an
 * asynchronous copy gave up records SPECTRAL_FAULT_WAIT_TIMEOUT and returns instead of hanging.
 * No counterpart in the reference, whose kernels have no waits. */
#define SPECTRAL_FAULT_WAIT_TIMEOUT 1u
#define SPECTRAL_FAULT_DRAIN_TIMEOUT 2u /* the wait for a copy still in flight also gave up */
SPECTRAL_API int spectral_device_faults(unsigned* faults, int clear);

/* Test hook for the bounded-wait path above (no counterpart in the reference). One CTA stages
 * 1 KiB from `src` into shared memory with one bulk copy completing on an mbarrier and waits for
 * it with the library's bounded wait, as the staged row kernel does, then writes the staged
 * bytes to `dst`. With missing_bytes > 0 (a multiple of 16, at most 1 MiB) the barrier expects
 * that many bytes more than the copy delivers, so the wait gives up after spin_limit polls and
 * records SPECTRAL_FAULT_WAIT_TIMEOUT; the probe then completes the missing bytes itself and
 * waits (bounded) for the real copy to land before returning. With missing_bytes == 0 it records
 * nothing. src and dst: 1 KiB each, 16-byte aligned. Nothing faults or waits without a limit. */
SPECTRAL_API int spectral_probe_bounded_wait(const void* src, void* dst, unsigned missing_bytes,
                                             unsigned spin_limit, void* stream);

/* --- registry (reference: csrc/fft/registry.hpp:14-51, csrc/torch/ops.cpp:422-438) --------- */

/* Number of implementations; their names by index, in registry order; index of a name or -1. */
SPECTRAL_API int spectral_impl_count(void);
SPECTRAL_API const char* spectral_impl_name(int index);
SPECTRAL_API int spectral_impl_find(const char* name);

/* The limits and capabilities of FftImpl (registry.hpp:14-25): largest single-kernel transform
 * (2D and pruned), largest 1D complex transform, largest real transform, whether it has a
 * strided column kernel and in-kernel pruning, and whether real transforms need `work`.
 * Any output pointer may be NULL. */
SPECTRAL_API int spectral_impl_limits(const char* impl, int* max_n, int* max_c2c_n, int* max_real_n,
                         int* has_columns, int* has_pruned, int* real_needs_work);

/* --- elementwise (reference: csrc/ops/scale.hpp, scale_c2c) ---------------------------------- */

/* y = alpha * x over `count` complex values. */
SPECTRAL_API int spectral_scale(const void* x, void* y, size_t count, float alpha, void* stream);

/* --- 1D (reference: csrc/fft/fft.hpp:13-49, C2cFn / R2cFn / C2rFn) --------------------------- */

/* `batch` transforms of n complex points, n a power of two up to the implementation's
 * max_c2c_n. Out of place: x and y must not overlap. */
SPECTRAL_API int spectral_c2c(const char* impl, const void* x, void* y, int n, long long batch, int inverse,
                 void* stream);

/* Real to complex: `batch` rows of n floats to rows of n/2 + 1 complex values, n a power of two
 * from 2 up to max_real_n. `work` holds spectral_real_workspace() complex values. */
SPECTRAL_API int spectral_r2c(const char* impl, const float* x, void* y, int n, long long batch, void* work,
                 void* stream);

/* Complex to real, the inverse of spectral_r2c divided by n; the imaginary parts of the zero and
 * n/2 frequencies are ignored, as in numpy and torch. */
SPECTRAL_API int spectral_c2r(const char* impl, const void* x, float* y, int n, long long batch, void* work,
                 void* stream);

/* Complex values of `work` that spectral_r2c / spectral_c2r need (0 for the engine variants,
 * which fuse the real-transform step into their kernels). */
SPECTRAL_API int spectral_real_workspace(const char* impl, int n, long long batch, size_t* count);

/* Column transforms (reference: ColumnsFn, fft.hpp:51-60): `slabs` row-major arrays of n rows by
 * `cols` columns, back to back; every column is an n-point transform. In place when x == y.
 * Only implementations with has_columns. */
SPECTRAL_API int spectral_columns(const char* impl, const void* x, void* y, int n, int cols, long long slabs,
                     int inverse, void* stream);

/* --- 2D (reference: csrc/fft/fft2d.hpp:27-39) ------------------------------------------------- */

SPECTRAL_API int spectral_fft2_c2c_workspace(const char* impl, int columns, int n1, int n2, long long batch,
                                size_t* count);
SPECTRAL_API int spectral_fft2_r2c_workspace(const char* impl, int columns, int n1, int n2, long long batch,
                                size_t* count);
SPECTRAL_API int spectral_fft2_c2r_workspace(const char* impl, int columns, int n1, int n2, long long batch,
                                size_t* count);

/* `batch` arrays of n1 x n2, rows then columns by `columns` (SPECTRAL_COLUMNS_*). */
SPECTRAL_API int spectral_fft2_c2c(const char* impl, int columns, const void* x, void* y, int n1, int n2,
                      long long batch, int inverse, void* work, void* stream);
/* Real (n1 x n2 floats) to complex (n1 x (n2/2 + 1)). */
SPECTRAL_API int spectral_fft2_r2c(const char* impl, int columns, const float* x, void* y, int n1, int n2,
                      long long batch, void* work, void* stream);
/* Complex (n1 x (n2/2 + 1)) to real (n1 x n2 floats), divided by n1 n2. */
SPECTRAL_API int spectral_fft2_c2r(const char* impl, int columns, const void* x, float* y, int n1, int n2,
                      long long batch, void* work, void* stream);

/* The complex-to-real 2D transform (strided columns) without any allocation, for callers that
 * cannot allocate device memory: a plugin whose host framework owns every allocation, a
 * real-time loop that must stay out of the CUDA allocator, or a binding that has device pointers
 * but no allocator. Its workspace is a fixed array inside the library of
 * SPECTRAL_NOALLOC_SCRATCH_VALUES complex values (32 MiB), held on every GPU that loads the
 * library until the process exits; larger transforms (batch * n1 * (n2/2 + 1) values) are
 * rejected with SPECTRAL_INVALID_ARGUMENT. All calls on a device share that array, so calls that
 * overlap on the GPU race and must be serialised by the caller. The first call on each device
 * looks up the array's device address; make it before any stream capture. Results equal
 * spectral_fft2_c2r with SPECTRAL_COLUMNS_STRIDED. No counterpart in the reference, which always
 * allocates its workspaces. */
#define SPECTRAL_NOALLOC_SCRATCH_VALUES (1u << 22)
SPECTRAL_API int spectral_fft2_c2r_noalloc(const char* impl, const void* x, float* y, int n1, int n2,
                                           long long batch, void* stream);

/* --- pruned, the FNO transforms (reference: csrc/fft/pruned.hpp:26-43) ------------------------ */

SPECTRAL_API int spectral_c2c_pruned_workspace(const char* impl, int n, int keep, long long batch, size_t* count);
/* Forward: the first `keep` of the n outputs per transform (x rows of n, y rows of keep).
 * Inverse: x rows of keep modes, the rest zero, to y rows of n, divided by n. */
SPECTRAL_API int spectral_c2c_pruned(const char* impl, const void* x, void* y, int n, int keep, long long batch,
                        int inverse, void* work, void* stream);

SPECTRAL_API int spectral_rfft2_modes_workspace(const char* impl, int n1, int n2, int m1, int m2,
                                   long long batch, size_t* count);
SPECTRAL_API int spectral_irfft2_modes_workspace(const char* impl, int n1, int n2, int m1, int m2,
                                    long long batch, size_t* count);
/* The (2 m1) x m2 low-frequency modes of each rfft2 of n1 x n2 real values: rows 0 .. m1-1, then
 * n1-m1 .. n1-1; columns 0 .. m2-1 (spectral.reference.rfft2_truncate). Out of place: x and
 * modes (and, for the inverse below, modes and y) must not overlap. */
SPECTRAL_API int spectral_rfft2_modes(const char* impl, const float* x, void* modes, int n1, int n2, int m1,
                         int m2, long long batch, void* work, void* stream);
/* spectral_rfft2_modes with the row stage's method chosen by the caller (no reference
 * counterpart):
 *   SPECTRAL_MODES_AUTO    what spectral_rfft2_modes uses;
 *   SPECTRAL_MODES_FP32    the FP32 FFT engine for rows and columns (one fused kernel);
 *   SPECTRAL_MODES_TENSOR  the rows as a GEMM with the kept DFT outputs on the tcgen05 tensor
 *                          cores, every FP32 operand split into two TF32 parts (three products
 *                          per multiply: FP32-level error); the columns by the FFT engine. Needs
 *                          an engine implementation, n1 = n2 = 128, m2 <= 16 and a 16-byte
 *                          aligned x; other shapes are refused. */
#define SPECTRAL_MODES_AUTO 0
#define SPECTRAL_MODES_FP32 1
#define SPECTRAL_MODES_TENSOR 2
SPECTRAL_API int spectral_rfft2_modes_method(const char* impl, const float* x, void* modes, int n1, int n2,
                                             int m1, int m2, long long batch, int method, void* work,
                                             void* stream);
/* The inverse: every other mode zero, then irfft2 (spectral.reference.irfft2_from_modes). */
SPECTRAL_API int spectral_irfft2_modes(const char* impl, const void* modes, float* y, int n1, int n2, int m1,
                          int m2, long long batch, void* work, void* stream);
/* spectral_irfft2_modes with the method chosen by the caller (no reference counterpart), as
 * spectral_rfft2_modes_method: SPECTRAL_MODES_TENSOR runs the columns by the FFT engine and each
 * real row as a GEMM with the kept columns' cosines and sines on the tcgen05 tensor cores (split
 * TF32). Needs an engine implementation, n1 = n2 = 128, m2 <= 16 and a 16-byte aligned y. */
SPECTRAL_API int spectral_irfft2_modes_method(const char* impl, const void* modes, float* y, int n1, int n2,
                                              int m1, int m2, long long batch, int method, void* work,
                                              void* stream);

/* --- the large single-field 2D transform, slab-decomposed over ranks --------------------------- */
/* An n x n complex field (n a power of two up to 16384) whose rows are split over `ranks` GPUs
 * (rank r holds rows r n/ranks ..), w = n / ranks. No counterpart in the reference: its fft2
 * stops at 4096 per side (csrc/fft/fft2d.cu:65-75) and it has no multi-GPU code.
 * Forward: spectral_slab_rows(x = the rank's rows x n, y = `ranks` chunks [s][row][c] of w
 * columns each), an all-to-all of those chunks (caller's NCCL), then spectral_slab_columns on
 * the received n x w matrix: the rank's w columns of the 2D transform, natural order.
 * Inverse (divided by n^2 overall): spectral_slab_columns(inverse) on the column slab, the
 * all-to-all of its row blocks, then spectral_slab_rows(inverse) from the received chunks. */
SPECTRAL_API int spectral_slab_rows(const void* x, void* y, int n, long long rows, int ranks,
                                    int inverse, void* stream);
/* (spectral_slab_rows is out of place: x and y, rows x n values each, must not overlap.)
 * n-point transforms down every column of the n x width row-major matrix x, into y (natural
 * order, same layout). x is used as scratch for n > 4096; x and y must not overlap. */
SPECTRAL_API int spectral_slab_columns(void* x, void* y, int n, int width, int inverse,
                                       void* stream);

/* The row stage with the exchange done in the same kernel through peer memory instead of an
 * all-to-all (no counterpart in the reference, which has no multi-GPU code). peers[s] (s = 0 ..
 * ranks-1, at most 8) is rank s's n x w column-slab buffer, mapped into this GPU's address space
 * (spectral_ipc_open; peers[rank] is this rank's own buffer). Forward: the row transforms of x
 * (this rank's rows x n) store chunk s of every row straight into peers[s], rows rank * rows ..;
 * y is unused. Inverse: the row transforms load chunk s of every row from peers[s] (the column
 * slabs after spectral_slab_columns(inverse)) and write this rank's rows to y; x is unused. The
 * ranks must be ordered around the call: every rank's writes (forward) or column stage (inverse)
 * complete before any rank reads them, e.g. by a collective on the same stream. */
SPECTRAL_API int spectral_slab_rows_peer(const void* x, void* y, void* const* peers, int n,
                                         long long rows, int rank, int ranks, int inverse,
                                         void* stream);

/* Natural layout. The column slab leaves rank r with output columns [r w, (r+1) w); a second
 * exchange of its w x w row blocks returns rows [r w, (r+1) w) of the transform instead. This
 * entry point copies, for each rank r (at most 16), the h x w block at src[r] (row stride
 * src_stride complex values) to dst[r] (row stride dst_stride); the 2D slab uses h = w. After the exchange of the column
 * slab's row blocks, src[r] = recv + r w^2 (stride w) and dst[r] = out + r w (stride n) give
 * the natural w x n rows. Before an inverse, src[r] = x + r w (stride n) and dst[r] = send +
 * r w^2 (stride w) pack the send blocks. src[r] may be another rank's buffer mapped through
 * CUDA IPC (plain NVLink loads), which fuses the exchange into the copy. */
/* No source block may share memory with any destination block (checked). */
SPECTRAL_API int spectral_slab_relayout(const void* const* src, void* const* dst, int ranks, int h, int w,
                                        long long src_stride, long long dst_stride, void* stream);

/* The 1D transform of n = n1 n2 points (n at most 2^24) distributed over ranks, each holding a
 * contiguous n / ranks of the signal (no counterpart in the reference, which has no multi-GPU
 * code). Viewing x as n1 rows by n2 columns, x[j1 n2 + j2]:
 *   1. the relayout packs the rank's rows into blocks of n1/R x n2/R; an all-to-all gives each rank
 *      the (n1, n2/R) slab of its columns j2 = col0 .. col0 + n2/R - 1;
 *   2. spectral_slab_twiddle_columns: n1-point transforms down that slab, output k1 multiplied by
 *      W_n^(k1 j2) (conjugate for the inverse, which also divides by n1);
 *   3. an all-to-all of the slab's row blocks and the relayout give the rank's n1/R rows k1;
 *   4. spectral_c2c: n2-point row transforms;
 *   5. the relayout packs the row blocks; an all-to-all gives each rank the (n1, n2/R) slab of
 *      its columns k2; spectral_transpose turns it into (n2/R, n1): X[k1 + n1 k2] for the rank's
 *      k2, its contiguous share of the output.
 * spectral_transpose: y = the transpose of `batch` row-major rows x cols arrays. */
SPECTRAL_API int spectral_slab_twiddle_columns(const void* x, void* y, int n1, int width, long long col0,
                                               long long n, int inverse, void* stream);
SPECTRAL_API int spectral_transpose(const void* x, void* y, int rows, int cols, long long batch, void* stream);

/* The whole slab transform through the C ABI, with the exchange on an NCCL communicator given as
 * void* (ncclComm_t; no counterpart in the reference). Forward: x is this rank's n/ranks rows
 * (rows x n), y receives its n x n/ranks column slab of fft2. Inverse: x is the column slab, y
 * receives the rank's rows of ifft2 (divided by n^2). work: spectral_fft2_slab_workspace
 * complex values. The library does not link NCCL: the entry points are resolved at run time
 * from the libnccl.so.2 already loaded into the process (else the one the loader finds), so a
 * communicator the caller made with its own NCCL works. spectral_slab_exchange is the exchange
 * alone (chunk s of send to rank s, chunk s of recv from rank s, values_per_rank complex values
 * each); spectral_nccl_* make and free a communicator for callers without NCCL of their own
 * (the SPECTRAL_NCCL_ID_BYTES-byte id from one rank, passed to every rank). */
#define SPECTRAL_NCCL_ID_BYTES 128
SPECTRAL_API int spectral_fft2_slab_workspace(int n, int ranks, size_t* count);
SPECTRAL_API int spectral_fft2_slab(const void* x, void* y, void* work, int n, int rank, int ranks,
                                    int inverse, void* comm, void* stream);
SPECTRAL_API int spectral_slab_exchange(const void* send, void* recv, long long values_per_rank, int ranks,
                                        void* comm, void* stream);
SPECTRAL_API int spectral_nccl_unique_id(void* id);
SPECTRAL_API int spectral_nccl_comm_init(const void* id, int rank, int ranks, void** comm);
SPECTRAL_API int spectral_nccl_comm_destroy(void* comm);

/* Device buffers shared between the processes of one node through CUDA IPC, for the buffers
 * spectral_slab_rows_peer addresses: allocate (cudaMalloc on the current device) and export a
 * SPECTRAL_IPC_HANDLE_BYTES-byte handle; map another process's handle (peer access enabled on
 * demand); unmap; free. */
#define SPECTRAL_IPC_HANDLE_BYTES 64
SPECTRAL_API int spectral_ipc_alloc(unsigned long long bytes, void** ptr, void* handle);
SPECTRAL_API int spectral_ipc_open(const void* handle, void** ptr);
SPECTRAL_API int spectral_ipc_close(void* ptr);
SPECTRAL_API int spectral_ipc_free(void* ptr);

/* --- per-mode channel contraction of an FNO spectral convolution --------------------------- */

/* out[b, o, m] = sum_i x[b, i, m] * w[i, o, m] over complex values: x (batch, cin, modes),
 * w (cin, cout, modes), out (batch, cout, modes), all contiguous. No reference counterpart: the
 * reference plans it (docs/ROADMAP.md:71-76, tasks 3.3-3.6) but has no implementation. */
SPECTRAL_API int spectral_mode_contract(const void* x, const void* w, void* out, long long batch, int cin,
                           int cout, long long modes, void* stream);

/* The same contraction with the method chosen by the caller (no reference counterpart):
 *   SPECTRAL_CONTRACT_AUTO    what spectral_mode_contract uses;
 *   SPECTRAL_CONTRACT_FP32    FP32 fused multiply-adds on the CUDA cores;
 *   SPECTRAL_CONTRACT_TENSOR  the tcgen05 tensor cores with every FP32 operand split into two TF32
 *                             parts (three products per multiply: FP32-level error). Needs batch
 *                             and cout multiples of 64, cin of 8, modes of 4, 16-byte aligned
 *                             arrays; other shapes are refused. */
#define SPECTRAL_CONTRACT_AUTO 0
#define SPECTRAL_CONTRACT_FP32 1
#define SPECTRAL_CONTRACT_TENSOR 2
SPECTRAL_API int spectral_mode_contract_method(const void* x, const void* w, void* out, long long batch,
                                               int cin, int cout, long long modes, int method, void* stream);

/* The FP32 arithmetic ceiling, for the roofline of FP32-bound kernels such as the contraction
 * (reference: csrc/tools/peaks.cu:46-70, a separate tool there). Launches one full wave of CTAs
 * that run independent fused multiply-add chains and nothing else: scalar FFMA (packed == 0) or
 * Blackwell's packed FP32x2 FFMA2 (packed != 0), `iters` trips of 128 chain steps per thread.
 * *flops receives the floating-point operations the launch performs (2 per FFMA, 4 per FFMA2);
 * the caller times the launch on `stream`. sink: one float, written only by a test the compiler
 * cannot fold (never true in practice). */
SPECTRAL_API int spectral_fp32_ceiling(float* sink, int iters, int packed, void* stream, double* flops);

/* --- radio signals: windowed spectrum and overlap-save FIR (reference: python/spectral/rf.py) -- */

/* Windowed spectrum of back-to-back frames (rf.py:94-102, spectrum): each of `rows` complex
 * signals of n samples (x, rows * n values) is cut into frames = max(1, ceil(n / nfft)) frames
 * of nfft samples, the last zero-padded; each frame is multiplied by `window` (nfft floats; NULL
 * for the rectangular window) and transformed. y: rows * frames * nfft values. nfft a power of
 * two from 2 to 4096; `impl` one of the stockham names (the others have no fused kernel). One
 * kernel: framing, padding and window are applied in the transform's load. */
SPECTRAL_API int spectral_spectrum(const char* impl, const void* x, const float* window, void* y, long long n,
                                   int nfft, long long rows, void* stream);

/* Causal FIR filter by overlap-save (rf.py:120-153, fir), y[j] = sum_k taps[k] x[j - k] with
 * zero initial state, per row of n samples: blocks of nfft samples overlapping by taps - 1, each
 * transformed, multiplied by taps_spectrum (the nfft-point forward transform of the taps zero-
 * padded to nfft, e.g. from spectral_c2c), transformed back; the last nfft - taps + 1 outputs of
 * each block are kept. x and y: rows * n values, not overlapping. nfft a power of two from
 * max(2, taps) to 4096; `impl` one of the stockham names. One kernel: both transforms and the
 * product run on chip. */
SPECTRAL_API int spectral_fir(const char* impl, const void* x, const void* taps_spectrum, void* y, long long n,
                              int nfft, int taps, long long rows, void* stream);

/* --- the Navier-Stokes solver's step stage (reference: python/spectral/flow/gpu.py:115-129) ---- */

/* One stage of the IMEX Crank-Nicolson / Heun step for `batch` vorticity spectra of an n x n grid
 * (n a power of two, 16 .. 512) in the pruned layout: 2m rows (ky = 0 .. m-1, then -m .. -1) by
 * m columns (kx = 0 .. m-1), complex values, 2 m <= n. With F(s) = forcing - mask * rfft2(u wx +
 * v wy) the dealiased tendency of state s (u, v, wx, wy the inverse transforms of s times the four
 * `derive` tables (4, 2m, m): i ky / |k|^2, -i kx / |k|^2, i kx, i ky):
 *   stage 0 (predictor): f0 = F(x),  out = (E w + dt f0) I          (x is w)
 *   stage 1 (corrector): out = (E w + dt/2 (f0 + F(x))) I           (x is the predictor's out)
 * forcing (2m, m) complex; mask (2m, m), explicit_factor E and implicit_factor I ((2m, m) or one
 * (2m, m) plane per trajectory: visc_stride 0 or 2 m m) float. out may be w for the corrector.
 * `work` holds spectral_flow_workspace() complex values. Three kernels, no physical field in
 * global memory; `impl` one of the stockham names. */
SPECTRAL_API int spectral_flow_workspace(int n, int m, long long batch, size_t* count);
SPECTRAL_API int spectral_flow_stage(const char* impl, const void* x, const void* w, void* f0, void* out,
                                     const void* derive, const void* forcing, const float* mask,
                                     const float* explicit_factor, const float* implicit_factor,
                                     long long visc_stride, void* work, int n, int m, long long batch,
                                     float dt, int stage, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SPECTRAL_B200_H */
