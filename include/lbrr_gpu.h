/*
 * lbrr_gpu.h -- C ABI of the B200 (sm_100a) BS-RoFormer engine.
 *
 * Drop-in for the GPU pipeline of logic-bs-roformer-rs (`lbrr`): everything
 * src/main.rs does from `CudaContext::new` to the device-to-host copy of the
 * separated stems, i.e. upload_weights (src/main.rs:6045-6077),
 * bench_forward + transformer_step (:7014-7162, :6131-6268), istft_ola
 * (:5024-5039) and the song loop with ola_demix (:7598-7775, :5052-5123).
 *
 * Conventions (modelled on the reference's own C shim,
 * tools/cudnn_sdpa_wrap.cpp:149-168, :226-244): opaque handles, int status
 * (0 = OK, negative = error), a thread-local last-error string, all device
 * work ordered on one stream per engine.  No function aborts or exits.  An
 * engine serves one host thread at a time; different engines may be driven
 * from different threads concurrently.
 * Plain pointers and sizes only; `stream` is a cudaStream_t passed as void*.
 *
 * Layouts at the boundary (src/main.rs:7283, :7739, src/benchmark.rs:93):
 *   input audio   interleaved stereo fp32 [len][2]
 *   output stems  planar fp32 [6][2][len], stem order of the model YAML
 *                 (bass, drums, other, vocals, guitar, piano)
 * fp16 tensors of the per-op entry points are IEEE binary16 bit patterns
 * (uint16_t), row-major.
 */
#ifndef LBRR_GPU_H
#define LBRR_GPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LBRR_OK 0
#define LBRR_ERR_INVALID (-1)       /* bad argument / shape / configuration           */
#define LBRR_ERR_CUDA (-2)          /* a CUDA runtime or cuFFT call failed             */
#define LBRR_ERR_WEIGHTS (-3)       /* checkpoint validation failed                    */
#define LBRR_ERR_DEVICE (-4)        /* a kernel reported a status (wait timeout, ...)  */
#define LBRR_ERR_STATE (-5)         /* call out of order (e.g. forward before weights) */
#define LBRR_ERR_PEER (-6)          /* multi-GPU stitching failed                      */

typedef struct lbrr_engine lbrr_engine;

/* Model hyper-parameters; replaces config.rs ModelConfig (src/config.rs:92-133).
 * The engine supports exactly the BS-RoFormer geometry of
 * assets/logic_bs_roformer.yaml and rejects anything else with LBRR_ERR_INVALID. */
typedef struct lbrr_model_desc {
  int32_t dim;            /* 256  */
  int32_t depth;          /* 12   */
  int32_t heads;          /* 8    */
  int32_t dim_head;       /* 64   */
  int32_t num_stems;      /* 6    */
  int32_t mlp_expansion;  /* 4    */
  int32_t n_fft;          /* 2048 */
  int32_t hop;            /* 512  */
  int32_t sample_rate;    /* 44100 */
  int32_t num_bands;      /* 62   */
  const int32_t* freqs_per_band; /* num_bands entries, sum 1025 */
} lbrr_model_desc;

/* One fp32 checkpoint tensor, keyed by its safetensors name (src/weights.rs:41-55). */
typedef struct lbrr_weight_view {
  const char* name;
  const float* data;      /* host memory, row-major as stored in the checkpoint */
  int64_t numel;
} lbrr_weight_view;

/* Song chunking.  The reference plan (src/main.rs:7617-7619, tools/bench_ref.py:
 * 13, :47-65): chunk 588800, step 559360, border 29440, linear fade of width
 * border.  BASELINE config 4's plan: chunk 588800, step 294400 (50 % overlap),
 * border 294400, Hann fade.  Either way the song is reflect-padded by `border`
 * on the left, each chunk's output y is accumulated as y * w with w * w into a
 * counter (the first chunk's leading and the last chunk's trailing `border`
 * samples weighted 1), and the sum is divided by max(counter, 1e-8). */
#define LBRR_FADE_LINEAR 0  /* w = ramps of width border at both chunk ends */
#define LBRR_FADE_HANN 1    /* w = periodic Hann window over the whole chunk */
typedef struct lbrr_chunk_plan {
  int64_t chunk;
  int64_t step;
  int64_t border;
  int64_t fade;   /* LBRR_FADE_LINEAR (0, a zero-initialised plan) or LBRR_FADE_HANN */
} lbrr_chunk_plan;

/* Last error message of the calling thread (replaces wrap_last_error,
 * tools/cudnn_sdpa_wrap.cpp:68, :244).  Never NULL. */
const char* lbrr_last_error(void);

/* ABI version: 2 (2 added lbrr_chunk_plan.fade, engine options and stage entry points). */
int lbrr_abi_version(void);

/* Page-locked host memory for the host entry points (lbrr_forward_chunk_host
 * copies straight between such buffers and the device): `bytes` of portable
 * page-locked memory in *ptr, released by lbrr_host_free.  No counterpart in
 * the reference, whose host buffers are ordinary Vec<f32>s staged by cudarc. */
int lbrr_host_alloc(size_t bytes, void** ptr);
int lbrr_host_free(void* ptr);

/* Fill `desc` with the supported model (assets/logic_bs_roformer.yaml:11-84).
 * `freqs_out` receives num_bands (62) entries and is referenced by desc. */
int lbrr_default_model(lbrr_model_desc* desc, int32_t* freqs_out, int32_t capacity);

/* Create an engine on `device` with scratch sized for chunks of up to
 * max_chunk_samples stereo samples (replaces CudaContext::new + make_bench_bufs +
 * RuntimeScratch::new, src/main.rs:7645-7684, :7169-7197, :5995-6002). */
int lbrr_engine_create(int device, const lbrr_model_desc* desc, int64_t max_chunk_samples, lbrr_engine** out);

/* Validate and upload a checkpoint (replaces ModelWeights::load + upload_weights,
 * src/weights.rs:307-447, src/main.rs:6045-6077): every one of the 1989 keys
 * exactly once with its exact size, per-layer qkv/out biases bit-equal to
 * linear_62_bias_0 / linear_64_bias_0, rotary freqs = 1/10000^(2i/64).
 * GEMM weights are rounded to fp16 (RNE, the src/fp16.rs bit contract). */
int lbrr_engine_load_weights(lbrr_engine* e, const lbrr_weight_view* views, size_t n);

/* Same, reading a .safetensors file (F32 tensors; src/weights.rs:25-55). */
int lbrr_engine_load_safetensors(lbrr_engine* e, const char* path);

/* Host-only checkpoint validation with exactly the checks of
 * lbrr_engine_load_weights (no device needed); replaces `lbrr --check-weights`
 * (src/main.rs:97, ModelWeights::load src/weights.rs:307-447). */
int lbrr_check_weights(const lbrr_weight_view* views, size_t n);

/* Host-only validation of a .safetensors file: header parse, F32 dtypes, byte
 * lengths, then lbrr_check_weights on its tensors. */
int lbrr_check_safetensors(const char* path);

/* One chunk, device buffers on the engine's device, stream-ordered on `stream`
 * (NULL = the engine's own stream; to order after work on the legacy default
 * stream pass cudaStreamLegacy).  x_dev: [len][2] fp32, stems_dev: [6][2][len]
 * fp32.  len must satisfy n_fft/2 < len <= max_chunk_samples (src/main.rs:7263).
 * Replaces bench_forward + istft_ola (src/main.rs:7014-7162, :7303-7306). */
int lbrr_forward_chunk(lbrr_engine* e, const float* x_dev, int64_t len, float* stems_dev, void* stream);

/* Multi-chunk batching (the bench_forward pass of src/main.rs:7014-7162 over
 * n_chunks chunks of the same len at once): x_dev: n_chunks x [len][2] fp32
 * one after another, stems_dev: n_chunks x [6][2][len] fp32.  Every stage
 * runs once over the frames of all chunks (the GEMMs, the mask estimator and
 * the frequency-axis attention see n_chunks * T frames; the time-axis
 * attention and its RoPE keep each chunk's frames apart), so each chunk's
 * stems are bit-identical to lbrr_forward_chunk on that chunk alone.  Needs
 * n_chunks * (len / 512 + 1) <= max_chunk_samples / 512 + 1 (an engine made
 * with max_chunk_samples >= n_chunks * len + (n_chunks - 1) * 512).  With
 * LBRR_OPT_FFT_BACKEND 1 or LBRR_OPT_DC_NYQUIST_IMAG set the chunks run one
 * forward each.  Replayed as a CUDA graph like lbrr_forward_chunk. */
int lbrr_forward_chunks(lbrr_engine* e, const float* x_dev, int64_t len, int32_t n_chunks, float* stems_dev,
                        void* stream);

/* End to end from host memory: copy x_host to the device, forward, copy the
 * stems back, synchronise, check the device status.  When both buffers are
 * page-locked (cudaHostAlloc, or cudaHostRegister over the whole range; the
 * first and last bytes are checked), the copies go directly between them and
 * the device, and each stem's download starts as soon as that stem's mask
 * and inverse transform are done, while the next stem is computed.
 * Otherwise x_host is staged through the engine's pinned memory
 * and the stems come back in slices that the engine's four host copy threads
 * (started by the first such call) move into stems_host as each arrives.
 * Replaces bench_forward plus the D2H of src/main.rs:7303-7317.
 * x_host: [len][2], stems_host: [6][2][len]. */
int lbrr_forward_chunk_host(lbrr_engine* e, const float* x_host, int64_t len, float* stems_host);

/* Front end and the first n_steps transformer axes only (n_steps in 0..24;
 * 0 = band-split output); writes the folded token tensor x[T*62][256] fp32
 * to x_out_dev.  Diagnostic stage boundary of the same pipeline
 * (the reference's --dump-trunk taps, src/main.rs:7055-7092). */
int lbrr_forward_trunk(lbrr_engine* e, const float* x_dev, int64_t len, int n_steps, float* x_out_dev,
                       void* stream);

/* Back end of the chunk forward only -- mask estimator (both grouped GEMMs,
 * tanh, GLU and the complex mask application), C2R and overlap-add -- rerun
 * on the engine's scratch from the last forward's final-norm output and
 * spectrum; len must equal that forward's.  Diagnostic stage boundary (the
 * reference's mask stage, src/main.rs:7111-7160) used to time the
 * MaskEstimator grouped GEMMs on their own. */
int lbrr_forward_back(lbrr_engine* e, int64_t len, float* stems_dev, void* stream);

/* Copy an internal buffer of the last forward to host memory (after syncing the
 * engine stream): "spec" [2][T][1025] complex64, "c2r" (masked spectra)
 * [12][T][1025] complex64, "pcm" [12][T][2048] fp32 (only after a forward
 * through the cuFFT back end), "x" [T*62][256] fp32,
 * "xb16" [62][T][256] fp16, "hidden" [6*62][T][1024] fp16.  `bytes` must not
 * exceed the buffer's size for the current length.  Diagnostic taps like the
 * reference's --dump-trunk dumps (src/main.rs:7055-7150). */
int lbrr_engine_read_buffer(lbrr_engine* e, const char* name, void* host_dst, int64_t bytes);

/* Synchronise the engine stream and check the device status word. */
int lbrr_engine_sync(lbrr_engine* e);

/* Engine options (lbrr_engine_set_option / lbrr_engine_get_option).
 *
 * LBRR_OPT_DC_NYQUIST_IMAG  0 (default) or 1.  The reference's mask_apply
 *   (src/main.rs:1776-1817) multiplies every bin by the complex mask, so the
 *   DC and Nyquist bins it hands to the C2R transform carry an imaginary part
 *   (the mask's, times the real spectrum value).  A C2R transform is only
 *   defined for Hermitian input, where those parts are zero, and torch.istft
 *   (the model definition the reference's golden gate targets) drops them.  0
 *   keeps those two bins real; 1 keeps the imaginary parts exactly as the
 *   reference's GPU path computes them; the inverse transform then runs
 *   through cuFFT, whose C2R consumes them as the reference's does.
 * LBRR_OPT_FFT_BACKEND  0 (default) or 1.  0: the in-house FFT kernels, the
 *   forward transform fused with framing, spectrum and band RMSNorm, the
 *   inverse fused with windowing, overlap-add and the envelope (no "frames"
 *   or "pcm" buffers).  1: cuFFT R2C/C2R between separate framing, band-norm
 *   and overlap-add kernels, the reference's decomposition
 *   (src/stft.rs:36-57, src/main.rs:7033-7040, :7154-7160).
 * LBRR_OPT_SONG_FAIL_CHUNK  -1 (default) or a chunk index.  Test hook of the
 *   song entry point: this engine's host thread fails with LBRR_ERR_STATE just
 *   before the forward of that chunk, so the abort path of lbrr_separate_song
 *   (the other engines stop, the call returns the error) can be tested
 *   without any device fault. */
#define LBRR_OPT_DC_NYQUIST_IMAG 1
#define LBRR_OPT_SONG_FAIL_CHUNK 2
#define LBRR_OPT_FFT_BACKEND 3
/* Read-only (lbrr_engine_get_option): kernels of this library launched by the
 * last chunk forward (cuFFT's own kernels not counted); a replayed CUDA graph
 * launches the same kernels. */
#define LBRR_INFO_KERNELS_PER_FORWARD 100
/* Read-only: host-side phase times, in microseconds, of the last weight load
 * (file read and header parse, both 0 for lbrr_engine_load_weights; validation
 * plus fp16 packing; the host-to-device copy) and of the last per-length setup
 * (RoPE and tile tables, FFT plans, ISTFT envelope), as the reference's
 * --bench JSON reports them (timing_ms, src/main.rs:7339-7343). */
#define LBRR_INFO_WEIGHTS_READ_US 101
#define LBRR_INFO_WEIGHTS_PARSE_US 102
#define LBRR_INFO_WEIGHTS_PACK_US 103
#define LBRR_INFO_WEIGHTS_H2D_US 104
#define LBRR_INFO_SETUP_US 105
int lbrr_engine_set_option(lbrr_engine* e, int option, int64_t value);
int lbrr_engine_get_option(const lbrr_engine* e, int option, int64_t* value);

/* Test of the bounded device waits (no counterpart in the reference, whose
 * waits are unbounded): launches on the engine stream one CTA that waits,
 * through the same bounded mbarrier wait every pipeline kernel uses, on a
 * barrier nothing completes, with a bound of limit_ns (1 ms .. 10 s).  No
 * asynchronous copy or MMA is in flight, so the CTA records the timeout in
 * the engine's status word and returns; the next lbrr_engine_sync reports
 * LBRR_ERR_DEVICE and clears the status, and the engine stays usable. */
int lbrr_engine_wait_probe(lbrr_engine* e, int64_t limit_ns);

/* Resident bytes: weights and scratch (src/main.rs:7199-7252). */
int lbrr_engine_memory(const lbrr_engine* e, int64_t* weight_bytes, int64_t* scratch_bytes);

void lbrr_engine_destroy(lbrr_engine* e);

/* Whole song (replaces separate()'s GPU loop, src/main.rs:7617-7775): reflect
 * pad, chunk grid, per-chunk forward, fade-weighted overlap-add, division by
 * the fade energy, crop.  Chunks are dealt round-robin over the n_engines
 * engines (one per GPU, one host thread each, each engine listed once).  With
 * the reference plan (chunks overlapping by less than half) every engine
 * finishes the song samples its chunks start, receiving only the previous
 * chunk's overlap strip from its neighbour engine (a device-to-device copy,
 * over NVLink between GPUs), and copies them to host_out itself; the result
 * is bit-identical to accumulating all chunks in order on one GPU, whatever
 * n_engines is.  Plans overlapping by half or more accumulate on engines[0].
 * host_interleaved: [len][2]; host_out: [6][2][len].  Either buffer may be
 * page-locked (lbrr_host_alloc, or any cudaHostAlloc / cudaHostRegister
 * range covering it): the engines then copy chunks in and finished regions
 * out by DMA straight from and into it instead of through their own pinned
 * staging buffers; the result is the same bits. */
int lbrr_separate_song(lbrr_engine* const* engines, int n_engines, const float* host_interleaved, int64_t len,
                       const lbrr_chunk_plan* plan, float* host_out);

/* ---------------------------------------------------------------------------
 * Per-op entry points (device pointers, fp16 as uint16_t bits).  Each mirrors
 * one kernel or library call of transformer_step / bench_forward and exists so
 * the pieces can be checked and timed on their own.  All are asynchronous on
 * `stream`; lbrr_op_sync() synchronises it and checks the per-device status.
 * ------------------------------------------------------------------------- */

/* rmsnorm_gates_h16 (src/main.rs:616-703): h16[rows][256], gates[rows][8]. */
int lbrr_op_norm_gates(const float* x, const float* gamma, const float* gate_w, const float* gate_b, uint16_t* h16,
                       float* gates, int64_t rows, void* stream);

/* QKV GEMM + shared bias (fp16) + RoPE on Q and K (cuBLASLt matmul_f16out +
 * rope_q16_inplace + rope_k16, src/main.rs:6157-6187).  h16[M][256],
 * w16[1536][256], bias16[1536] (fp32 values already rounded to fp16),
 * cos/sin[P][32] with P = frames (axis 0) or bands (axis 1), qkv[M][1536],
 * M = frames * bands, token = t*bands + b. */
int lbrr_op_qkv_rope(const uint16_t* h16, const uint16_t* w16, const float* bias16, const float* cos_tab,
                     const float* sin_tab, uint16_t* qkv, int64_t frames, int32_t bands, int32_t axis, void* stream);

/* Gated SDPA over one axis (CudnnSdpa::execute + sdpa_gate,
 * src/main.rs:6193-6199): out[M][512] = f16(f16(softmax(QK^T/8) V) * sigmoid(gate)). */
int lbrr_op_attention(const uint16_t* qkv, const float* gates, uint16_t* out, int64_t frames, int32_t bands,
                      int32_t axis, void* stream);

/* Out-projection + bias + residual, fused with the pre-FF RMSNorm
 * (matmul_resid + rmsnorm_h16, src/main.rs:6219-6234). */
int lbrr_op_outproj_norm(const uint16_t* scaled16, const uint16_t* w16, const float* bias, const float* resid,
                         const float* gamma, float* attn_out, uint16_t* h16, int64_t rows, void* stream);

/* FF1 + A&S-erf GELU, fp16 out (gemm_f16_gelu_a16w, src/main.rs:2827-2949). */
int lbrr_op_ff1_gelu(const uint16_t* h16, const uint16_t* w16, const float* b1, uint16_t* ff1, int64_t rows,
                     void* stream);

/* FF2 + bias + residual (matmul_resid, src/main.rs:6255-6259). */
int lbrr_op_ff2_resid(const uint16_t* ff1, const uint16_t* w16, const float* b2, const float* resid, float* x,
                      int64_t rows, void* stream);

/* Feed-forward in one kernel: x = FF2(f16(gelu(FF1(h16) + b1))) + b2 + resid,
 * the same values as lbrr_op_ff1_gelu followed by lbrr_op_ff2_resid
 * (src/main.rs:6234-6259) without the [rows][1024] fp16 intermediate in
 * device memory.  w1_16 [1024][256], w2_16 [256][1024] fp16. */
int lbrr_op_feed_forward(const uint16_t* h16, const uint16_t* w1_16, const float* b1, const uint16_t* w2_16,
                         const float* b2, const float* resid, float* x, int64_t rows, void* stream);

int lbrr_op_sync(void* stream);

/* Feed-forward half of a RoFormer step (FF1 + GELU, then FF2 + bias +
 * residual into x) that allocates no device memory; it has no counterpart in
 * the reference.  For callers that cannot call cudaMalloc: a real-time audio
 * host calling from its render thread, or an application that gives the
 * library a fixed device-memory budget.  The fp16 hidden activations use a
 * file-scope static device array of 8192 x 1024 halves (16 MiB, held by every
 * GPU that loads the library until exit); rows > 8192 are rejected with
 * LBRR_ERR_INVALID.  The first call on a device (with that device current)
 * resolves the array's address, loads the library's kernels on the device and
 * sets their attributes, so it may block: make it once per device as a
 * warm-up, outside any real-time thread.  Every call synchronises `stream`
 * before it returns (it reads the kernels' status back and reports a nonzero
 * one as LBRR_ERR_DEVICE), so calls cannot be recorded into a CUDA graph.  Do
 * not call it again after cudaDeviceReset of that device.  Calls share the
 * array: work of calls that overlaps on the GPU races.  Shapes: h16 [rows][256], w1 [1024][256],
 * b1 [1024], w2 [256][1024], b2 [256], resid and x [rows][256] fp32. */
int lbrr_op_feed_forward_noalloc(const uint16_t* h16, const uint16_t* w1_16, const float* b1, const uint16_t* w2_16,
                                 const float* b2, const float* resid, float* x, int64_t rows, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* LBRR_GPU_H */
