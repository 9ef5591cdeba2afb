#pragma once

/*
 * welvet_b200.h -- additive entry points of libwelvet_b200.so. None of these exists in the
 * reference; they extend its Dense-session ABI (include/welvet_c.h:81-86) with device
 * pointers, CUDA streams, a native-bytes mount, persistent SwiGLU / MHA cells, a device-
 * resident volume chain and the codec kernels, without changing any reference symbol.
 *
 * Device-pointer calls run asynchronously on the given stream (`stream` is a cudaStream_t;
 * 0 is the legacy default stream, as everywhere in CUDA) and must not overlap another call
 * on the same session. Host-pointer calls are synchronous like the reference ABI.
 */

#include "welvet_c.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Library build identifier, e.g. "welvet-b200 0.1 sm_100a". */
WELVET_API const char* welvet_b200_build_id(void);

/* ---------------------------------------------------------------- Dense */

/* Like welvet_dense_mount, with W_dev a device pointer to the float32 matrix (no H2D copy
 * of the unquantized weights). bias stays a host pointer. */
WELVET_API welvet_status welvet_b200_dense_mount_device(int32_t batch, int32_t in, int32_t out,
                                                        int32_t act, int32_t dtype, const float* W_dev,
                                                        const double* bias, size_t bias_len,
                                                        welvet_dense_session** sess_out);

/* Mount from a FormatNone store already packed in the reference layout (native bytes and
 * per-tensor scale, e.g. read back from an NWS1 snapshot). */
WELVET_API welvet_status welvet_b200_dense_mount_native(int32_t batch, int32_t in, int32_t out,
                                                        int32_t act, int32_t dtype,
                                                        const uint8_t* native, size_t native_len,
                                                        float scale, const double* bias,
                                                        size_t bias_len,
                                                        welvet_dense_session** sess_out);

/* Forward with device pointers: x_dev [batch][in], pre_dev/post_dev [batch][out]. */
WELVET_API welvet_status welvet_b200_dense_execute_device(welvet_dense_session* sess,
                                                          const float* x_dev, float* pre_dev,
                                                          float* post_dev, void* stream);

/* No counterpart in the reference (which runs one session per call, src/interop/c_abi.cpp
 * welvet_dense_execute). n independent forwards on one stream: sessions i = 0..n-1 read
 * x_dev[i] and write pre_dev[i] / post_dev[i] (device pointers, as in
 * welvet_b200_dense_execute_device). Sessions that share dtype, shape and batch (1..4) and
 * run the small-batch tensor GEMV go out in grouped launches of up to 32 layers, one kernel
 * over all of them; otherwise each session runs on its own. Asynchronous on `stream`. */
WELVET_API welvet_status welvet_b200_dense_execute_group_device(welvet_dense_session* const* sessions, int32_t n,
                                                                const float* const* x_dev,
                                                                float* const* pre_dev,
                                                                float* const* post_dev, void* stream);

/* No counterpart in the reference. welvet_b200_dense_execute_device without any allocation,
 * for callers that cannot call cudaMalloc while they run a forward: a serving loop that must
 * not stall on an allocation (cudaMalloc can synchronize the device), or a framework or
 * plugin host that owns all device memory up front and forbids allocations afterwards. It runs
 * the batched tensor-core forward (a session of batch > 8, FP8/FP4/Int8, outside exact mode;
 * other sessions get status 2) with the scratch of that kernel -- x split into f16 planes,
 * per-token scales, split-K partials -- in one static 32 MiB device array that the library
 * holds on every GPU that loads it until the process exits; a call needing more returns
 * status 1. The first call on a device (and the first after that device's context was
 * re-created) looks up the array's device address. All calls share the array: calls whose
 * kernels overlap on one GPU (other streams
 * or threads) race and must be serialized by the caller. A timed-out pipeline wait is
 * recorded in the session's error word, which welvet_b200_dense_check_error reads. */
WELVET_API welvet_status welvet_b200_dense_execute_device_noalloc(welvet_dense_session* sess,
                                                                  const float* x_dev, float* pre_dev,
                                                                  float* post_dev, void* stream);

/* No counterpart in the reference (whose calls are all synchronous). Synchronizes `stream`
 * and reports, then clears, a pipeline wait of the batched tensor-core kernel that timed out
 * in an earlier asynchronous call on this session (execute_device, execute_device_noalloc):
 * status 4 if one did, 0 otherwise. Copies 4 bytes to the host; allocates nothing. */
WELVET_API welvet_status welvet_b200_dense_check_error(welvet_dense_session* sess, void* stream);

/* No counterpart in the reference. The launch plan of the batched tensor-core GEMM (the TMEM
 * kernel) for a layer of `rows` outputs x `cols` inputs at M tokens, with at most `xsplit`
 * f16 planes of x and token blocks capped at `max_tb` (0: no cap), as the library plans it
 * before a launch: host arithmetic only, no device call, for checks and tuning. The
 * WELVET_B200_GEMM_* environment switches apply; a CTA-pair plan is reported as planned,
 * before the launch asks the device whether pairs fit. out[0..n) receives, in this order:
 * pair, TB, tpass[3], nacc[3], acc_cols, acc_buf, a_col, sx, sw, x_bytes, w_bytes, smem,
 * nkb, splits, kb_per_split, tiles_t, tiles, tail_first, tail_s, tail_kbps, n_items. Returns
 * the number of values in a plan (25) whatever n is, or -1 for a dtype the GEMM does not
 * serve or a non-positive size. */
WELVET_API int32_t welvet_b200_gemm_plan(int32_t M, int32_t cols, int32_t rows, int32_t xsplit, int32_t dtype,
                                         int32_t max_tb, int64_t* out, int32_t n);

/* The session's authoritative host store: dtype, rows (= out), cols (= in), scale and the
 * native bytes in the reference layout (FP4: low nibble = even flat index). Float32 stores
 * return their float payload. *native_len is always set; the bytes are copied when
 * cap >= *native_len. */
WELVET_API welvet_status welvet_b200_dense_store(welvet_dense_session* sess, int32_t* dtype,
                                                 int32_t* rows, int32_t* cols, float* scale,
                                                 uint8_t* native_out, size_t cap,
                                                 size_t* native_len);

/* ---------------------------------------------------------------- codecs (device buffers) */

/* FormatNone encode of n float32 values (device) to reference-layout bytes (device) and the
 * per-tensor scale (device float). Bit-exact with the reference host codec. */
WELVET_API welvet_status welvet_b200_codec_encode(int32_t dtype, const float* w_dev, int64_t n,
                                                  uint8_t* native_dev, float* scale_dev,
                                                  void* stream);
/* Reference-semantics decode of n elements (device) to float32 (device). */
WELVET_API welvet_status welvet_b200_codec_decode(int32_t dtype, const uint8_t* native_dev,
                                                  int64_t n, float scale, float* out_dev,
                                                  void* stream);
/* Exhaustive-encode digest: sum over float32 bit patterns i in [start, start+count) of
 * splitmix64((i << 8) | code(i)) mod 2^64; codec 0 = E4M3, 1 = E5M2, 2 = FP4. Synchronous. */
WELVET_API welvet_status welvet_b200_codec_digest(int32_t codec, uint64_t start, uint64_t count,
                                                  uint64_t* digest);
/* Every code through the GEMV's vector decoders (after device canonicalisation):
 * FP4 -> 512 floats (256 bytes, low nibble first), FP8E4M3/FP8E5M2/Int8 -> 256 floats. */
WELVET_API welvet_status welvet_b200_codec_selftest_decode(int32_t dtype, float* out_host);

/* ---------------------------------------------------------------- SwiGLU cell */

typedef struct welvet_b200_swiglu welvet_b200_swiglu;
/* Gate/Up [intermediate x input], Down [input x intermediate] float32; weights_on_device
 * selects device or host pointers. */
WELVET_API welvet_status welvet_b200_swiglu_mount(int32_t input_dim, int32_t intermediate_dim,
                                                  int32_t dtype, const float* Gate, const float* Up,
                                                  const float* Down, int32_t weights_on_device,
                                                  welvet_b200_swiglu** out);
/* rows = batch*seq. h_dev [rows][intermediate] may be NULL; y_dev [rows][input]. */
WELVET_API welvet_status welvet_b200_swiglu_execute_device(welvet_b200_swiglu* s, int32_t rows,
                                                           const float* x_dev, float* h_dev,
                                                           float* y_dev, void* stream);
WELVET_API void welvet_b200_swiglu_release(welvet_b200_swiglu* s);

/* ---------------------------------------------------------------- MHA cell */

typedef struct welvet_b200_mha welvet_b200_mha;
WELVET_API welvet_status welvet_b200_mha_mount(int32_t d_model, int32_t num_heads,
                                               int32_t num_kv_heads, int32_t head_dim,
                                               int32_t max_seq_len, int32_t mask, int32_t pos,
                                               int32_t dtype, const float* Q, const float* K,
                                               const float* V, const float* O,
                                               int32_t weights_on_device, welvet_b200_mha** out);
/* x_dev [batch*seq][d_model] -> attn_dev [batch*seq][q_dim] (may be NULL), y_dev [..][d_model]. */
WELVET_API welvet_status welvet_b200_mha_execute_device(welvet_b200_mha* s, int32_t batch,
                                                        int32_t seq, const float* x_dev,
                                                        float* attn_dev, float* y_dev, void* stream);
WELVET_API void welvet_b200_mha_release(welvet_b200_mha* s);

/* ---------------------------------------------------------------- volume (Grid) */

/* A depth x rows x cols x layers_per_cell grid of cells (reference architecture::Grid,
 * include/welvet/architecture.hpp:100-141; non-positive dimensions become 1) run in hop order
 * z, y, x, l with activations kept on the device (reference runtime::forward::volume_dense,
 * src/runtime/forward.cpp:98-156). Coordinates out of range return status 1. */
typedef struct welvet_b200_volume welvet_b200_volume;
WELVET_API welvet_status welvet_b200_volume_create(int32_t depth, int32_t rows, int32_t cols,
                                                   int32_t layers_per_cell, welvet_b200_volume** out);
WELVET_API welvet_status welvet_b200_volume_bind_dense(welvet_b200_volume* v, int32_t z, int32_t y,
                                                       int32_t x, int32_t l, int32_t in, int32_t out,
                                                       int32_t act, int32_t dtype, const float* W,
                                                       const double* bias, size_t bias_len,
                                                       int32_t weights_on_device);
WELVET_API welvet_status welvet_b200_volume_bind_dense_native(welvet_b200_volume* v, int32_t z,
                                                              int32_t y, int32_t x, int32_t l,
                                                              int32_t in, int32_t out, int32_t act,
                                                              int32_t dtype, const uint8_t* native,
                                                              size_t native_len, float scale,
                                                              const double* bias, size_t bias_len);
WELVET_API welvet_status welvet_b200_volume_bind_swiglu(welvet_b200_volume* v, int32_t z, int32_t y,
                                                        int32_t x, int32_t l, int32_t input_dim,
                                                        int32_t intermediate_dim, int32_t dtype,
                                                        const float* Gate, const float* Up,
                                                        const float* Down, int32_t weights_on_device);
WELVET_API welvet_status welvet_b200_volume_bind_mha(welvet_b200_volume* v, int32_t z, int32_t y,
                                                     int32_t x, int32_t l, int32_t d_model,
                                                     int32_t num_heads, int32_t num_kv_heads,
                                                     int32_t head_dim, int32_t max_seq_len,
                                                     int32_t mask, int32_t pos, int32_t seq,
                                                     int32_t dtype, const float* Q, const float* K,
                                                     const float* V, const float* O,
                                                     int32_t weights_on_device);
WELVET_API welvet_status welvet_b200_volume_bind_rmsnorm(welvet_b200_volume* v, int32_t z, int32_t y,
                                                         int32_t x, int32_t l, int32_t dim, double eps,
                                                         int32_t dtype, const float* gamma);
/* reference architecture::set_remote_link (src/architecture/grid.cpp:97-107) */
WELVET_API welvet_status welvet_b200_volume_set_remote_link(welvet_b200_volume* v, int32_t z, int32_t y,
                                                            int32_t x, int32_t l, int32_t tz,
                                                            int32_t ty, int32_t tx, int32_t tl);
WELVET_API welvet_status welvet_b200_volume_set_disabled(welvet_b200_volume* v, int32_t z, int32_t y,
                                                         int32_t x, int32_t l, int32_t disabled);
WELVET_API int32_t welvet_b200_volume_hops(welvet_b200_volume* v);
/* Runs hops [hop_begin, hop_end) (-1 = to the end) on `rows` rows of x_dev [rows][in_width];
 * the last executed cell's post goes to out_dev (may be NULL), its width to *out_width. */
WELVET_API welvet_status welvet_b200_volume_forward_device(welvet_b200_volume* v, int32_t rows,
                                                           const float* x_dev, int32_t in_width,
                                                           int32_t hop_begin, int32_t hop_end,
                                                           float* out_dev, int32_t* out_width,
                                                           void* stream);
/* Host-buffer forward over every hop, synchronous. out_host receives the last executed cell's
   post densely as [rows][*out_width]; out_cap is its capacity in floats. */
WELVET_API welvet_status welvet_b200_volume_forward_f32(welvet_b200_volume* v, int32_t rows,
                                                        const float* x_host, int32_t in_width,
                                                        float* out_host, size_t out_cap,
                                                        int32_t* out_width);
/* Device pointers of a cell's last pre / post ([rows][width]), for per-step records. */
WELVET_API welvet_status welvet_b200_volume_cell_outputs(welvet_b200_volume* v, int32_t z, int32_t y,
                                                         int32_t x, int32_t l, const float** pre,
                                                         int32_t* pre_width, const float** post,
                                                         int32_t* post_width);
WELVET_API void welvet_b200_volume_release(welvet_b200_volume* v);

/* ---------------------------------------------------------------- multi-GPU (one box)
 *
 * No counterpart in the reference, which runs every kernel on device 0
 * (src/cuda/device.cpp:40-61). One process per GPU; the processes of a job form a
 * communicator (NCCL, loaded at run time: libnccl.so.2, or the path in WELVET_B200_NCCL).
 * Collective calls (marked so) must be made by every rank, in the same order. */

typedef struct welvet_b200_comm welvet_b200_comm;
/* 1 when NCCL could be loaded into this process, else 0 (the comm calls then return 2). */
WELVET_API int32_t welvet_b200_nccl_available(void);
/* A new job id (ncclGetUniqueId): 128 bytes that rank 0 makes and hands to every rank. */
WELVET_API welvet_status welvet_b200_comm_unique_id(uint8_t* id128);
/* Collective: this process becomes `rank` of `nranks` on CUDA device `device`. */
WELVET_API welvet_status welvet_b200_comm_create(const uint8_t* id128, int32_t nranks, int32_t rank,
                                                 int32_t device, welvet_b200_comm** out);
WELVET_API void welvet_b200_comm_release(welvet_b200_comm* c);

/* Output rows [*begin, *end) that `rank` holds of a column-sharded layer with `rows` outputs:
 * whole 128-row blocks dealt in rank order (host arithmetic only). */
WELVET_API welvet_status welvet_b200_shard_rows(int32_t rows, int32_t nranks, int32_t rank, int32_t* begin,
                                                int32_t* end);
/* Hops [*hop_begin, *hop_end) of a volume of `cells` cells x `layers_per_cell` that `rank` runs
 * in the cell-per-GPU pipeline: whole cells, contiguous in hop order (host arithmetic only). */
WELVET_API welvet_status welvet_b200_stage_plan(int32_t cells, int32_t layers_per_cell, int32_t nranks,
                                                int32_t rank, int32_t* hop_begin, int32_t* hop_end);

/* A Dense layer (in -> out) too large for one GPU, split by output rows over the ranks of
 * `comm`: this rank passes its rows W_rows [end - begin][in] (welvet_b200_shard_rows; host or
 * device pointer per weights_on_device) and the whole layer's bias (host, rows o < bias_len).
 * mode 0: each rank's kernels store its columns of the output straight into every rank's
 * output buffer over NVLink peer memory, then the ranks exchange one flag each; mode 1: local
 * forward, then ncclAllGather and a permute (the library baseline). Collective. */
typedef struct welvet_b200_sharded_dense welvet_b200_sharded_dense;
WELVET_API welvet_status welvet_b200_sharded_dense_mount(welvet_b200_comm* comm, int32_t batch, int32_t in,
                                                         int32_t out, int32_t act, int32_t dtype,
                                                         const float* W_rows, int32_t weights_on_device,
                                                         const double* bias, size_t bias_len, int32_t mode,
                                                         welvet_b200_sharded_dense** s);
/* Collective. One forward of x_dev [batch][in] (the same x on every rank), asynchronous on
 * `stream`: *post_dev receives the library-owned device buffer holding the whole output
 * [batch][out] on this rank once the stream gets there, *pre_dev that of pre -- the same
 * buffer for a Linear layer without bias, else a buffer with this rank's columns of pre (the
 * others zero). The buffers of one call stay valid until the call after next. */
WELVET_API welvet_status welvet_b200_sharded_dense_execute_device(welvet_b200_sharded_dense* s,
                                                                  const float* x_dev, void* stream,
                                                                  const float** post_dev,
                                                                  const float** pre_dev);
/* Collective, synchronous: host x [batch][in] in, host pre / post [batch][out] out (either may
 * be NULL), like welvet_dense_execute. */
WELVET_API welvet_status welvet_b200_sharded_dense_execute(welvet_b200_sharded_dense* s, const float* x,
                                                           float* pre, float* post);
/* Synchronizes `stream`; status 4 if a rank did not reach an output exchange within the wait
 * limit (WELVET_B200_SHARD_WAIT_MS, default 5000) or a tensor-core pipeline wait timed out. */
WELVET_API welvet_status welvet_b200_sharded_dense_check_error(welvet_b200_sharded_dense* s, void* stream);
/* This rank's output rows. */
WELVET_API welvet_status welvet_b200_sharded_dense_rows(welvet_b200_sharded_dense* s, int32_t* row_begin,
                                                        int32_t* row_end);
WELVET_API void welvet_b200_sharded_dense_release(welvet_b200_sharded_dense* s);

/* Collective. The cell-per-GPU pipeline of a volume forward (reference
 * runtime::forward::volume_dense, src/runtime/forward.cpp:98-156, placed over GPUs): this rank
 * runs hops [hop_begin, hop_end) (welvet_b200_stage_plan) of `v` on micro-batches of `micro`
 * rows; rank 0 reads x_dev [rows][stage_in_width], every other rank receives its stage input
 * (width stage_in_width) from the rank before and sends its stage output to the rank after
 * (NCCL point-to-point); the last rank's output is broadcast, so out_dev [rows][out_width]
 * holds the volume's output on every rank. Rows are independent through the cells, so the
 * result equals the one-GPU forward of the same micro-batches. Remote links must stay within
 * a rank's hops. Asynchronous on `stream`. */
WELVET_API welvet_status welvet_b200_volume_pipeline_forward_device(welvet_b200_volume* v, welvet_b200_comm* comm,
                                                                    int32_t hop_begin, int32_t hop_end, int32_t rows,
                                                                    const float* x_dev, int32_t stage_in_width,
                                                                    int32_t micro, float* out_dev,
                                                                    int32_t out_width, void* stream);

#ifdef __cplusplus
}
#endif
