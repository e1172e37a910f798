/*
 * nsc_b200.h -- C ABI of the B200 (sm_100a) shift-window kernel library
 * `libnsc_b200.so`.
 *
 * This ABI replaces the pybind11 module `neural_shift_cuda._C` of the
 * reference project (csrc/shift_ops.cpp:347-368, csrc/metropolis.cpp:42-48).
 * Differences from that module, all deliberate:
 *   - plain device pointers and int64 extents, no torch types;
 *   - outputs and scratch are allocated by the caller; the library never
 *     allocates device memory and never synchronizes;
 *   - the shift table is a HOST pointer to S rows of `shift_cols` int64
 *     values (dx, dy[, has_inv]); it is copied into the kernel parameters;
 *     has_inv 0 = no mirror term, 1 = masked mirror (the reference's
 *     meaning), 2 = periodic mirror (extension, accumulate / normalized:
 *     the mirror term reads (p - d) mod (H, W) with no inside test; not
 *     accepted by the row-band entry points), 3 = transposed row
 *     (extension, accumulate_uz only: the row adds w_s(p - d) x(p - d)
 *     read circularly and no forward term -- K^T of the forward-only row
 *     without a rolled copy of the weight plane);
 *   - inputs keep their storage dtype (fp16/bf16/fp32 are read natively and
 *     promoted in registers; fp64 stays fp64) instead of being copied to a
 *     promoted tensor first;
 *   - a weight stack may be channel-broadcast (`w_channels == 1` while
 *     C > 1): it is read once per pixel and applied to every channel.
 *
 * Layouts: images (B, C, H, W); weight stacks (S*B, w_channels, H, W) for
 * accumulate / normalized; (B, S, w_channels, H, W) for metropolis; all
 * contiguous row-major.  `stream` is a cudaStream_t (NULL = legacy default).
 * Every call is asynchronous on `stream` and uses the current device.
 * Errors: a non-zero nsc_status; nsc_last_error_string() gives the message
 * for the calling host thread.
 */
#ifndef NSC_B200_H
#define NSC_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define NSC_API __attribute__((visibility("default")))
#else
#define NSC_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum nsc_status {
    NSC_OK = 0,
    NSC_ERR_INVALID_ARG = 1,       /* shape / pointer / shift-table error */
    NSC_ERR_UNSUPPORTED_DTYPE = 2, /* dtype or dtype combination */
    NSC_ERR_S_OUT_OF_RANGE = 3,    /* S outside [1, 1024] */
    NSC_ERR_LAUNCH_FAILED = 4,     /* cudaGetLastError after a launch */
    NSC_ERR_TIMEOUT = 5            /* a bounded device-side wait gave up */
} nsc_status;

typedef enum nsc_dtype {
    NSC_F16 = 0,
    NSC_BF16 = 1,
    NSC_F32 = 2,
    NSC_F64 = 3
} nsc_dtype;

/* ABI marker; replaces `_C.index_width_bits()` (csrc/shift_ops.cpp:351).
 * Always 64: shifts and flattened offsets are int64 end to end. */
NSC_API int nsc_index_width_bits(void);

/* Library version string ("0.12.0-b200.N"). */
NSC_API const char* nsc_version(void);

/* Message of the last failed call on this host thread ("" if none). */
NSC_API const char* nsc_last_error_string(void);

/* Number of bounded device-side waits (mbarrier polls in the tiled
 * kernels) that gave up on the current device since the library loaded;
 * 0 in a healthy run.  A kernel whose wait gives up stops waiting and
 * returns instead of hanging, leaving its outputs undefined.  This call
 * synchronizes with the device (a diagnostic, not for hot loops); it
 * returns 0xFFFFFFFF if the counter cannot be read. */
NSC_API unsigned int nsc_wait_timeouts(void);

/* Synchronizes `stream` and returns NSC_ERR_TIMEOUT when bounded device
 * waits of the current device gave up since the previous nsc_check_waits
 * on that device (the kernels concerned returned early; their outputs are
 * undefined), NSC_OK otherwise.  No counterpart in the reference (whose
 * kernels have no waits); the host-side status of the bounded-wait design. */
NSC_API nsc_status nsc_check_waits(void* stream);

/* Test hook, no counterpart in the reference: subsequent tiled
 * accumulate / normalized launches leave weight copy number `skip_copy`
 * (per CTA, counted from 0; -1 = none) unissued and give every bounded
 * wait `wait_budget` hinted sleeps of about 1 ms (0 = the default of
 * 4096).  With a skipped copy the consumers' waits on it run out, the
 * kernel returns early and nsc_check_waits reports NSC_ERR_TIMEOUT; the
 * context stays usable.  Reset with nsc_test_wait_fault(-1, 0). */
NSC_API void nsc_test_wait_fault(int skip_copy, unsigned int wait_budget);

/* ---------------------------------------------------------------------
 * Gathers.  Replace shift_gather_forward / pair_gather_forward
 * (csrc/shift_ops.cpp:81-140) and their backward (shift_ops.cpp:102-156).
 * out : (S*B, C, H, W) for shift_gather, (S*B, 2C, H, W) for pair_gather,
 *       same dtype as guide (bit-exact copies);
 * mask: (S*B, 1, H, W) in guide dtype, 1 where (h+dx, w+dy) is inside.
 * Backward: grad_out in the forward output layout -> grad_guide (B,C,H,W),
 * same dtype, accumulated in fp32 (fp64 for fp64), deterministic.
 * shift_cols is 2 or 3 (only dx, dy are read).
 * ------------------------------------------------------------------- */
NSC_API nsc_status nsc_shift_gather_fwd(const void* guide, int dtype,
                                int64_t B, int64_t C, int64_t H, int64_t W,
                                const int64_t* shifts, int64_t S,
                                int64_t shift_cols, void* out, void* mask,
                                void* stream);
NSC_API nsc_status nsc_pair_gather_fwd(const void* guide, int dtype,
                               int64_t B, int64_t C, int64_t H, int64_t W,
                               const int64_t* shifts, int64_t S,
                               int64_t shift_cols, void* out, void* mask,
                               void* stream);
NSC_API nsc_status nsc_shift_gather_bwd(const void* grad_out, int dtype,
                                int64_t B, int64_t C, int64_t H, int64_t W,
                                const int64_t* shifts, int64_t S,
                                int64_t shift_cols, void* grad_guide,
                                void* stream);
NSC_API nsc_status nsc_pair_gather_bwd(const void* grad_out, int dtype,
                               int64_t B, int64_t C, int64_t H, int64_t W,
                               const int64_t* shifts, int64_t S,
                               int64_t shift_cols, void* grad_guide,
                               void* stream);

/* ---------------------------------------------------------------------
 * accumulate_uz.  Replaces accumulate_uz_forward / _backward
 * (csrc/shift_ops.cpp:160-212).  shifts: (S, 3).
 * x dtype / w dtype: equal, or x fp32 with w fp16/bf16; fp64 only with
 * fp64.  U, Z, grad_x: fp32 (fp64 for fp64 inputs); grad_U, grad_Z in
 * that same accumulator dtype.  grad_w: w's dtype and shape
 * (S*B, w_channels, H, W); a broadcast weight receives the channel sum.
 * ------------------------------------------------------------------- */
NSC_API nsc_status nsc_accumulate_uz_fwd(const void* x, int x_dtype,
                                 const void* w, int w_dtype,
                                 int64_t w_channels,
                                 int64_t B, int64_t C, int64_t H, int64_t W,
                                 const int64_t* shifts, int64_t S,
                                 void* U, void* Z, void* stream);
NSC_API nsc_status nsc_accumulate_uz_bwd(const void* x, int x_dtype,
                                 const void* w, int w_dtype,
                                 int64_t w_channels,
                                 int64_t B, int64_t C, int64_t H, int64_t W,
                                 const int64_t* shifts, int64_t S,
                                 const void* grad_U, const void* grad_Z,
                                 void* grad_x, void* grad_w, void* stream);

/* Row-band form of nsc_accumulate_uz_fwd for an image split into bands
 * of rows across devices.  The caller owns output rows [row0, row0+Hb) of
 * an image with Hg rows.  x_ext holds Hb + 2R rows: global rows
 * row0-R .. row0+Hb+R-1, already wrapped circularly; w holds the band's
 * Hb rows of every weight plane.  Mirror terms whose source pixel lies
 * outside the band are NOT added here (the owner of that row adds them,
 * see nsc_accumulate_uz_band_edges).  U, Z: (B, C, Hb, W). */
NSC_API nsc_status nsc_accumulate_uz_band_fwd(const void* x_ext, int x_dtype,
                                      const void* w, int w_dtype,
                                      int64_t w_channels, int64_t B,
                                      int64_t C, int64_t Hb, int64_t W,
                                      int64_t row0, int64_t Hg,
                                      const int64_t* shifts, int64_t S,
                                      void* U, void* Z, void* stream);

/* nsc_accumulate_uz_band_fwd restricted to the band's output rows
 * [r_begin, r_end) (other rows of U, Z are not written), with the
 * persistent grid capped at max_ctas CTAs (0: one per SM).  No counterpart
 * in the reference (which has no multi-GPU split): the interior rows
 * [R, Hb - R) read no halo row, so they run while the halo exchange is in
 * flight, on SMs left free for the collective; the 2R border rows follow
 * the exchange. */
NSC_API nsc_status nsc_accumulate_uz_band_rows_fwd(const void* x_ext, int x_dtype,
                                           const void* w, int w_dtype,
                                           int64_t w_channels, int64_t B,
                                           int64_t C, int64_t Hb, int64_t W,
                                           int64_t row0, int64_t Hg,
                                           int64_t r_begin, int64_t r_end,
                                           int max_ctas, const int64_t* shifts,
                                           int64_t S, void* U, void* Z,
                                           void* stream);

/* Mirror contributions of this band's own weights to the R rows just
 * above (edge_top: global rows row0-R .. row0-1) and just below
 * (edge_bot: rows row0+Hb .. row0+Hb+R-1) the band.  edge_top / edge_bot
 * are (2, B, C, R, W) accumulators (U part then Z part, fp32/fp64; R <= 32),
 * overwritten.  Rows outside the image [0, Hg) receive zeros. */
NSC_API nsc_status nsc_accumulate_uz_band_edges(const void* x_ext, int x_dtype,
                                        const void* w, int w_dtype,
                                        int64_t w_channels, int64_t B,
                                        int64_t C, int64_t Hb, int64_t W,
                                        int64_t row0, int64_t Hg,
                                        const int64_t* shifts, int64_t S,
                                        void* edge_top, void* edge_bot,
                                        void* stream);

/* Adds the neighbours' mirror strips to a band's (U, Z) in one launch:
 * strip_above (the upper band's edge_bot, may be NULL) onto rows 0 .. R-1,
 * strip_below (the lower band's edge_top, may be NULL) onto rows
 * Hb-R .. Hb-1.  acc_dtype: NSC_F32 or NSC_F64 (the type of U, Z and the
 * strips).  No reference counterpart (part of the row-band split). */
NSC_API nsc_status nsc_accumulate_uz_band_add_strips(void* U, void* Z, int acc_dtype,
                                             int64_t B, int64_t C, int64_t Hb,
                                             int64_t W, int64_t R,
                                             const void* strip_above,
                                             const void* strip_below,
                                             void* stream);

/* ---------------------------------------------------------------------
 * normalized_accumulate_uz.  Replaces normalized_accumulate_uz_forward /
 * _backward (csrc/shift_ops.cpp:218-283).  One pass per output with an
 * online running max.  log_weights != 0: weights are logits, -inf masks.
 * D, log_C: fp32 (fp64), shape (B, C, H, W).  Empty rows give D = 0,
 * log_C = -inf; NaN / +inf / negative-positive-weight rows give NaN.
 * invalid_flag (nullable, device int): the forward ORs 1 into it when a
 * weight breaks the contract (NaN or +inf; negative in positive mode),
 * which replaces the reference's separate validation pass (ops.py:209-224).
 * ------------------------------------------------------------------- */
NSC_API nsc_status nsc_normalized_accumulate_uz_fwd(
    const void* x, int x_dtype, const void* w, int w_dtype,
    int64_t w_channels, int64_t B, int64_t C, int64_t H, int64_t W,
    const int64_t* shifts, int64_t S, int log_weights,
    void* D, void* log_C, int* invalid_flag, void* stream);
NSC_API nsc_status nsc_normalized_accumulate_uz_bwd(
    const void* x, int x_dtype, const void* w, int w_dtype,
    int64_t w_channels, int64_t B, int64_t C, int64_t H, int64_t W,
    const int64_t* shifts, int64_t S, int log_weights,
    const void* D, const void* log_C, const void* grad_D,
    const void* grad_log_C, void* grad_x, void* grad_w, void* stream);

/* ---------------------------------------------------------------------
 * NECTR model-1 patched forward, fused.  Replaces the pair_gather ->
 * weight head -> normalized_accumulate_uz sequence of the reference's
 * NECTR installer (neural_shift_cuda/integration/nectr_patch.py:214-234,
 * ops pair_gather and normalized_accumulate_uz) for inference, without the
 * (S*B, 2L, H, W) pair batch.  The first 1x1 convolution of the head,
 * W1 [g(p); g(p+d)] + b1, is passed split: AB_map (B, 2 width, H, W) holds
 * W1[:, :L] g in channels [0, width) and W1[:, L:] g in [width, 2 width);
 * it is in `dtype` (fp32 or fp64), as is x (B, C, H, W), C in {1, 3}.
 * `params` (host, `n_params` doubles): b1[width]; LayerNorm-1 gamma[width],
 * beta[width]; for depth 2 also W2[width/2][width], b2[width/2],
 * LayerNorm-2 gamma, beta [width/2]; then the output convolution
 * Wout[cout][last width] (no bias), cout = C (mode 0, 1) or 3C (mode 2:
 * chunks k, a, b).  width in {8, 16, 32}, depth in {1, 2}, LeakyReLU
 * slope in [0, 1].
 * mode 1: exp head, logits v * inv_sigma2 (log weights); mode 2:
 * controlled sigmoid softplus(a) / (1 + exp(-sigmoid(b) k)) + 1e-8
 * (positive weights); mode 0: raw v with plain sums.  Forward keys are
 * masked by the box (p + d inside), mirror keys (has_inv rows) by p - d
 * inside.  out0/out1: D and log_C (modes 1, 2) or U and Z (mode 0),
 * (B, C, H, W) in `dtype`; `invalid_flag` (device int, may be NULL) is
 * OR-ed with 1 when a key is NaN / +inf (negative in mode 2).  Radius
 * <= 16 and (2 width + C)(8 + 2R)(32 + 2R) elements must fit in 227 KB of
 * shared memory.  No backward: the installer uses it when autograd is off.
 * ------------------------------------------------------------------- */
NSC_API nsc_status nsc_nectr_fused_fwd(const void* x, const void* AB_map,
                               int dtype, int64_t B,
                               int64_t C, int64_t H, int64_t W,
                               int64_t width, int depth,
                               const double* params, int64_t n_params,
                               double ln_eps1, double ln_eps2, double slope,
                               double inv_sigma2, const int64_t* shifts,
                               int64_t S, int mode, void* out0, void* out1,
                               int* invalid_flag, void* stream);

/* ---------------------------------------------------------------------
 * metropolis_aggregate.  Replaces `_C.metropolis_aggregate`
 * (csrc/metropolis.cpp:29-37, metropolis_cuda.cu:195-240) and adds the
 * backward the reference lacks.  w_half: (B, S, w_channels, H, W);
 * img: (B, C, H, W) same dtype class as w_half.  Wx, d_hat: img dtype.
 * degree: caller scratch (B, w_channels, H, W) in the accumulator dtype
 * (fp32, fp64 for fp64); the forward writes the raw degree d = K e there
 * and the backward reads it back.  grad_degree: caller scratch of the same
 * size for the backward.  grad_w: w_half's dtype and shape; grad_img:
 * img's dtype.
 * ------------------------------------------------------------------- */
NSC_API nsc_status nsc_metropolis_fwd(const void* w_half, int w_dtype,
                              int64_t w_channels, const void* img,
                              int x_dtype, int64_t B, int64_t C, int64_t H,
                              int64_t W, const int64_t* shifts, int64_t S,
                              int use_box, double eps, void* Wx, void* d_hat,
                              void* degree, void* stream);
NSC_API nsc_status nsc_metropolis_bwd(const void* w_half, int w_dtype,
                              int64_t w_channels, const void* img,
                              int x_dtype, int64_t B, int64_t C, int64_t H,
                              int64_t W, const int64_t* shifts, int64_t S,
                              int use_box, double eps, const void* degree,
                              const void* d_hat, const void* grad_Wx,
                              const void* grad_d_hat, void* grad_degree,
                              void* grad_w, void* grad_img, void* stream);

/* ---------------------------------------------------------------------
 * Allocation-free metropolis forward.  No counterpart in the reference.
 *
 * For callers that cannot allocate device memory: a plugin whose host
 * framework owns every allocation and hands it only the input and output
 * buffers (no workspace), or code that must not call cudaMalloc because
 * it can synchronize the device or fail in the middle of a run.  Same
 * arguments and results as nsc_metropolis_fwd, minus `degree`: the degree
 * map lives in a fixed scratch array inside the library instead.
 *
 * Limit: B * w_channels * H * W * sizeof(accumulator) must not exceed
 * NSC_NOALLOC_SCRATCH_BYTES (16 MiB: 4,194,304 fp32 values, e.g. 16 images
 * of 512 x 512 with channel-shared weights); larger calls fail with
 * NSC_ERR_INVALID_ARG.  The array is static device memory, held by every
 * GPU that loads the library until the process exits.  The first call on
 * a device looks the array's device address up (once per device); make
 * that first call before any stream capture.  Every call shares the one
 * array, so calls that overlap on the GPU (other streams, other threads)
 * race; serialize them.  The array keeps the last call's contents, which
 * is harmless: the degree pass overwrites every value it later reads.
 * ------------------------------------------------------------------- */
#define NSC_NOALLOC_SCRATCH_BYTES (16u << 20)
NSC_API nsc_status nsc_metropolis_fwd_noalloc(const void* w_half, int w_dtype,
                                      int64_t w_channels, const void* img,
                                      int x_dtype, int64_t B, int64_t C,
                                      int64_t H, int64_t W,
                                      const int64_t* shifts, int64_t S,
                                      int use_box, double eps, void* Wx,
                                      void* d_hat, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NSC_B200_H */
