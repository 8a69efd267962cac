/*
 * efg.h - C ABI of EdgeForge-B200: the packed Q4_0/Q8_0 matrix-product path of
 * EdgeForge (MG782469/EdgeForge) rebuilt for NVIDIA B200 (sm_100a).
 *
 * Conventions
 *  - Every function returns an int status (EFG_OK = 0, codes in efg_status.h below),
 *    except the few that return a value and document how they report errors.
 *    Nothing throws across this boundary. efg_last_error() gives a thread-local
 *    message for the most recent failure on the calling thread.
 *  - Pointers named d_* (and every pointer of the *_async / stream-taking calls) are
 *    DEVICE pointers (cudaMalloc or equivalent) on the current CUDA device. `stream` is
 *    a cudaStream_t passed as void* (NULL = the legacy default stream). Those calls are
 *    stream-ordered and return once the work is queued.
 *  - Calls with host_ in their name take HOST pointers and are synchronous: they are
 *    the reference's own signatures (include/ef/qkernels.h, include/ef/quant.h) with a
 *    status code added.
 *  - Storage types use the reference's numbering (ef::QType, include/ef/quant.h:35).
 *  - Block layout is the reference's, byte for byte (include/ef/quant.h:22-33):
 *      Q4_0: 18 bytes / 32 weights = fp16 d, then 16 bytes; byte j holds code j in its
 *            low nibble and code j+16 in its high nibble; w = (code - 8) * d.
 *      Q8_0: 34 bytes / 32 weights = fp16 d, then 32 int8 codes; w = code * d.
 *    A matrix is row-major [rows][cols] with rows packed back to back, exactly as
 *    stored in an .efq file (include/ef/qfile.h:1-21). cols must be a multiple of 32.
 *  - Device-side waits are bounded: a kernel that gives up records EFG_ETIMEOUT in a
 *    per-device error word, read (and cleared) with efg_device_error().
 */
#ifndef EFG_H
#define EFG_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (mirrors edgeforge_b200/csrc/efg_status.h) ------------------ */
#define EFG_OK 0
#define EFG_EINVAL 1
#define EFG_ECUDA 2
#define EFG_ENCCL 3
#define EFG_ETIMEOUT 4
#define EFG_ENOMEM 5
#define EFG_EFORMAT 6
#define EFG_ESTATE 7

/* ---- storage types: ef::QType (include/ef/quant.h:35) -------------------------- */
#define EFG_F32 0
#define EFG_F16 1
#define EFG_BF16 2
#define EFG_Q8_0 3
#define EFG_Q4_0 4

/* ABI version of this header; bumped on any incompatible change. */
int efg_abi_version(void);

/* Message of the last failure on this thread ("" if none). Replaces the what() of
 * ef::Error (include/ef/error.h:11-13). */
const char* efg_last_error(void);

/* Name of a status code ("EFG_OK", "EFG_EINVAL", ...). */
const char* efg_status_string(int status);

/* Reads and clears the error word that device-side bounded waits write on the current
 * device (synchronises the device first). *code receives EFG_OK or EFG_ETIMEOUT. */
int efg_device_error(int* code);

/* Early weight streaming for the matvec calls made afterwards on this thread (default
 * off). When on, a matvec may start copying its weight tiles while the previous kernel
 * in the stream is still running (programmatic dependent launch); it still waits for
 * that kernel before touching x or y. Only valid when W is not written by the kernels
 * just before it, which holds for model weights loaded once. Returns the old setting. */
int efg_set_weight_prefetch(int enable);

/* Which kernel computes the Q4_0 matvec calls made afterwards on this thread for large
 * matrices (48 MB and more, 2048 <= cols <= 8192, cols % 256 == 0, 16-byte aligned W, x
 * and norm weights). 1 (the default): the integer tensor-core kernel, exact int8 x int8
 * products of the codes and a 30-bit fixed-point x, which keeps HBM busier than the
 * CUDA-core kernel can on B200. 0: the CUDA-core kernel for every size. Both meet the
 * reference's tolerance (test_qinfer.cpp:58-67). Returns the old setting. No reference
 * counterpart: the reference has one CPU kernel per format. */
int efg_set_q4_mma(int enable);

/* Whether the Q4_0 GEMM calls made afterwards on this thread with B <= 64 columns use the
 * small-batch kernel on the exact integer MMA (X columns as int8 digit planes against the
 * codes) instead of the tcgen05 kernel. 0 (the default) keeps the tcgen05 kernel. Both meet the
 * same tolerance; the small-batch kernel also gives non-finite columns exactly as the FP32
 * matvec does. Returns the old setting. No reference counterpart. */
int efg_set_small_gemm(int enable);

/* Bytes of one row of `cols` weights, or 0 with efg_last_error() set when a block type
 * gets cols % 32 != 0. Replaces ef::qtype_row_bytes (include/ef/quant.h:42,
 * src/quant.cpp:136-149), which throws in that case. */
uint64_t efg_row_bytes(int qtype, uint64_t cols);

/* ================================================================ matvec
 * y[r] = dot(row r of W, x) for r < rows, FP32 activations and accumulation, read
 * straight from the packed blocks (no dequantized copy). Results agree with the
 * reference's scalar kernel within 1e-5 of sum_i |w_i x_i| per row (the reference's own
 * metric, tests/test_qinfer.cpp:58-67); the summation order differs, so not bit for bit.
 * Deterministic: the same inputs give the same bits on every call. y must not alias
 * x or W.
 */

/* Replaces ef::kern::matvec_q4_0 (include/ef/qkernels.h:50, src/qkernels.cpp:67-70). */
int efg_matvec_q4_0(float* d_y, const uint8_t* d_W, const float* d_x, size_t rows, size_t cols, void* stream);
/* Replaces ef::kern::matvec_q8_0 (include/ef/qkernels.h:51, src/qkernels.cpp:72-75). */
int efg_matvec_q8_0(float* d_y, const uint8_t* d_W, const float* d_x, size_t rows, size_t cols, void* stream);
/* Replaces ef::kern::matvec(y, WeightView, x, pool) (include/ef/qkernels.h:66,
 * src/qkernels.cpp:275-278) for every storage type: the packed EFG_Q4_0 / EFG_Q8_0 as above,
 * and EFG_F32 / EFG_F16 / EFG_BF16 rows of `cols` plain values (src/qkernels.cpp:237-269; a
 * tied BF16 lm_head, src/model.cpp:88,273), within the same 1e-5 of sum|w x|. */
int efg_matvec(int qtype, float* d_y, const uint8_t* d_W, const float* d_x, size_t rows, size_t cols, void* stream);

/* One job of a fused multi-matrix matvec: ef::kern::MatvecJob plus the WeightView it
 * points to (include/ef/qkernels.h:28-34,70-74). */
typedef struct {
  float* d_y;
  int qtype;
  const uint8_t* d_W;
  size_t rows, cols;
  const float* d_x;
} efg_matvec_job;

/* Replaces ef::kern::matvec_jobs (include/ef/qkernels.h:75, src/qkernels.cpp:280-297):
 * several products in one launch where the jobs share x, type and cols (q/k/v, gate/up);
 * otherwise one launch per job. Each job's rows are computed exactly as by efg_matvec. */
int efg_matvec_jobs(const efg_matvec_job* jobs, size_t n_jobs, void* stream);

/* Replaces ef::kern::dot_q4_0 / dot_q8_0 (include/ef/qkernels.h:47-48): *d_out = dot of
 * one packed row of n weights with x. */
int efg_dot_q4_0(float* d_out, const uint8_t* d_row, const float* d_x, size_t n, void* stream);
int efg_dot_q8_0(float* d_out, const uint8_t* d_row, const float* d_x, size_t n, void* stream);

/* ================================================================ quantize / dequantize
 * Bit-exact with the reference for every input, NaN and inf included.
 */

/* Replaces ef::quantize_row (include/ef/quant.h:52, src/quant.cpp:182-218) for
 * EFG_Q4_0 (search != 0: the MSE scale search + least-squares refinement of
 * src/quant.cpp:26-99; 0: the absmax scale), EFG_Q8_0 (search ignored) and the plain
 * conversions EFG_F32 (the bits), EFG_F16 and EFG_BF16 (round to nearest even, the
 * reference's NaN rules; any n). */
int efg_quantize_row(int qtype, const float* d_x, size_t n, void* d_out, int search, void* stream);
/* Replaces ef::fake_quant_q4_group (include/ef/quant.h:58, src/quant.cpp:243-248): the Q4
 * quantize -> dequantize of one group of n values with one FP16 scale (the scale search of
 * q4_group when search != 0); only the first min(n, 256) values are written, as in the
 * reference. Bit-exact. */
int efg_fake_quant_q4_group(const float* d_x, size_t n, float* d_out, int search, void* stream);
/* Replaces ef::dequantize_row (include/ef/quant.h:53, src/quant.cpp:220-249) for the
 * block types, and EFG_F32/EFG_F16/EFG_BF16 (exact widening). */
int efg_dequantize_row(int qtype, const void* d_in, size_t n, float* d_out, void* stream);
/* [rows][cols] forms of the two calls above: the loop of quantize_tensor_rows
 * (src/quantizer.cpp:121-149) over a whole matrix in one launch. */
int efg_quantize_rows(int qtype, const float* d_X, size_t rows, size_t cols, void* d_out, int search, void* stream);
int efg_dequantize_rows(int qtype, const void* d_in, size_t rows, size_t cols, float* d_out, void* stream);

/* Replaces ef::kern::row_f32 (include/ef/qkernels.h:78, src/qkernels.cpp:299-305):
 * row r of W as FP32 (embedding lookup). r is read from device memory (*d_r) when
 * d_r is not NULL, else r_host is used. */
int efg_row_f32(float* d_out, int qtype, const uint8_t* d_W, size_t rows, size_t cols, const int32_t* d_r,
                size_t r_host, void* stream);

/* ================================================================ host-pointer forms
 * Synchronous calls with the reference's exact arguments (host pointers). x is copied in
 * and y out on every call. W is read from a resident device copy when it lies inside a
 * range registered with efg_host_register_weights() (the reference passes read-only
 * views of a memory-mapped .efq, src/model.cpp:71-74: register the file's data once at
 * load); otherwise it is uploaded on every call, so a caller that rewrites its buffer
 * between calls always gets results for the current bytes. A page-locked y (cudaHostAlloc,
 * cudaHostRegister, torch pin_memory) is written by the matvec kernel's own stores over the
 * bus, saving a separate device-to-host copy per call; pageable y, and page-locked y that
 * the device may not write (registered with cudaHostRegisterReadOnly), is copied after it.
 */
int efg_host_matvec(int qtype, float* y, const uint8_t* W, const float* x, size_t rows, size_t cols);
int efg_host_quantize_row(int qtype, const float* x, size_t n, void* out, int search);
int efg_host_fake_quant_q4_group(const float* x, size_t n, float* out, int search);
int efg_host_dequantize_row(int qtype, const void* in, size_t n, float* out);
/* Uploads [host, host + bytes) once and keeps it on the device; the caller promises not to
 * modify those bytes while registered. Registering a range again refreshes its copy. */
int efg_host_register_weights(const void* host, size_t bytes);
/* Drops the resident copy of the range starting at `host`. */
int efg_host_unregister_weights(const void* host);
/* Drops every resident copy. */
int efg_host_release_weights(void);

/* efg_host_matvec without device allocation: x, y and W are staged through one static
 * 8 MiB device area (its address taken once per device by the first call, which must come
 * before any stream capture); calls needing more than the area are rejected (EFG_EINVAL).
 * Every device has its own copy of the area: calls that overlap on the same device race on
 * it and must be serialized by the caller; calls on different devices do not. This entry
 * point has no reference counterpart: the reference's kern::matvec_q4_0/q8_0 allocate
 * nothing because they run on host memory. */
int efg_host_matvec_static(int qtype, float* y, const uint8_t* W, const float* x, size_t rows, size_t cols);

/* ================================================================ batched GEMM (tensor cores) */

/* Y[b][m] = sum_k W[m][k] X[b][k] for b < B: the matvec of every column of a batch at once,
 * on the tcgen05 tensor cores (W dequantized to an exact BF16 hi+lo pair, X split into two
 * BF16 parts, FP32 accumulation in TMEM). Layout: W packed Q4_0 [M] rows, X FP32 [B][K]
 * (each column contiguous, 16-byte aligned), Y FP32 [B][M]. The reference has no GEMM; it
 * runs ef::kern::matvec (qkernels.h:66) once per column, which each Y column matches
 * within 1e-5 of sum|w x| for finite inputs. For B > 64 the split X goes through one
 * per-device scratch: such calls on different streams must not overlap. An infinite x or FP16 scale splits into an
 * infinite high part and a NaN residual, so an output the matvec gives as +-inf comes out
 * NaN here (NaN outputs stay NaN). */
int efg_gemm_q4_0(float* d_Y, const uint8_t* d_W, const float* d_X, size_t M, size_t K, size_t B, void* stream);

/* The same product for Q8_0 weights: W dequantized to an exact sum of three BF16 terms (a
 * Q8_0 weight q d has up to 18 significant bits), K a multiple of 256, W and X 16-byte
 * aligned. Replaces B calls of ef::kern::matvec_q8_0 (qkernels.h:63-64) with one launch. */
int efg_gemm_q8_0(float* d_Y, const uint8_t* d_W, const float* d_X, size_t M, size_t K, size_t B, void* stream);

/* One launch for 1-3 matrices of one type (EFG_Q4_0 or EFG_Q8_0) that share X: Y_j = W_j X
 * for W_j of M[j] rows, or Y_j += W_j X when `accumulate` (fl(Y + product), bit-identical to
 * adding the product afterwards). K a multiple of 256 (K = 0 gives Y = 0, or Y unchanged when
 * adding; B = 0 and jobs of M = 0 rows do nothing), weights and X 16-byte aligned. The
 * decoder's fused q/k/v projection (kern::matvec_jobs, src/model.cpp:230) and the o / down
 * projections with their residual adds (src/model.cpp:247-249, 260-262), for a batch. */
int efg_gemm_jobs(int qtype, int n_jobs, const uint8_t* const* d_W, float* const* d_Y, const size_t* M,
                  const float* d_X, size_t K, size_t B, int accumulate, void* stream);

/* ================================================================ row-sharded matvec (several GPUs) */

/* A communicator between the GPUs of one node, one rank per GPU and process (or thread).
 * The library loads NCCL (libnccl.so.2) on first use. */
typedef struct efg_comm efg_comm;

/* Rows [*begin, *begin + *count) of a rows-row matrix belong to `rank` of `nranks`: the
 * contiguous split of ef::ThreadPool::chunk_begin (include/ef/threadpool.h:52-54). */
int efg_shard_rows(size_t rows, int nranks, int rank, size_t* begin, size_t* count);
/* Writes a fresh 128-byte NCCL unique id to `id` (made on one rank, given to all). */
int efg_comm_unique_id(void* id);
/* Joins the communicator `id` as `rank` of `nranks` on the current device (collective). */
int efg_comm_init(const void* id, int nranks, int rank, efg_comm** out);
int efg_comm_destroy(efg_comm* comm);
/* Registers d_buf (`bytes`, device memory from cudaMalloc or a caching allocator built on
 * it, on the communicator's device) so that the peers' kernels can store into it directly.
 * Collective: every rank calls it with its own buffer of the same size, and all ranks get
 * the same outcome (EFG_ECUDA on every rank when one cannot export or map its buffer, e.g.
 * several ranks in one process). At most 8 ranks. The exchange of handles uses the
 * communicator's NCCL; afterwards no library call is needed to move data. */
int efg_comm_register(efg_comm* comm, void* d_buf, size_t bytes);
/* Drops a registration (every rank calls it for its buffer; synchronises the device). */
int efg_comm_deregister(efg_comm* comm, void* d_buf);
/* Row-sharded ef::kern::matvec (qkernels.h:66) for a matrix too large for one GPU's share:
 * d_W_shard holds this rank's rows (efg_shard_rows) of the full [rows][cols] packed matrix,
 * d_x the whole x; on return (stream-ordered) d_y holds all `rows` outputs on every rank.
 * When d_y lies in a buffer registered with efg_comm_register (at the same offset on every
 * rank) and rows >= the rank count, the matvec kernel itself stores every output into every
 * rank's y over NVLink and finishes once all ranks' rows have arrived (one launch, no
 * collective call); every rank must then make the same sequence of these calls, and a rank
 * that waits more than 2 s for a peer records EFG_ETIMEOUT (efg_device_error), after which
 * the communicator must be destroyed. Otherwise the slices are exchanged in place through
 * NCCL (one all-gather, or one broadcast per rank when the split is uneven). Every rank calls
 * it with the same rows/cols. EFG_ENCCL on a collective failure. */
int efg_matvec_sharded(int qtype, float* d_y, const uint8_t* d_W_shard, const float* d_x, size_t rows, size_t cols,
                       efg_comm* comm, void* stream);
/* ef::kern::argmax (src/kernels.cpp:105-111) on the device: *d_index = the index of the
 * first maximum of d_x[0..n) (NaN never wins, except that a NaN at index 0 is kept; 0 for
 * n = 0). Stream-ordered. */
int efg_argmax(const float* d_x, size_t n, int32_t* d_index, void* stream);
/* The lm_head and the greedy argmax of the decode step (src/model.cpp:266-270, 278-304)
 * with lm_head row-sharded over the GPUs of one node: d_W_shard holds this rank's rows
 * (efg_shard_rows) of the [rows][cols] packed lm_head, d_x the whole hidden state and
 * d_norm_w (or NULL) the final RMSNorm weights. Writes this rank's logits (its row count of
 * floats) to d_logits_shard and, on every rank, the argmax over all rows (the rule of
 * efg_argmax) to *d_token: each rank reduces its logits to one (value, index) pair and the
 * pairs are exchanged. While any buffer is registered on the communicator
 * (efg_comm_register; all ranks share the outcome) the argmax launch itself stores its pair
 * into every rank's flag area over NVLink and waits (bounded, EFG_ETIMEOUT via
 * efg_device_error) for the peers' pairs: two launches per call and no collective; every rank
 * must then make the same sequence of these calls. Otherwise the pairs travel in one
 * 8-byte-per-rank NCCL all-gather. Every rank calls it with the same rows/cols. No
 * reference counterpart for the sharding itself. */
int efg_lm_head_argmax_sharded(int qtype, float* d_logits_shard, int32_t* d_token, const uint8_t* d_W_shard,
                               const float* d_x, const float* d_norm_w, float eps, size_t rows, size_t cols,
                               efg_comm* comm, void* stream);

/* ================================================================ .efq and the decode step */

/* Validates an .efq file image in memory: magic, version, JSON header, tensor table (types,
 * shapes, 64-byte offsets, bounds, overlaps), the exact tensor set the config requires and
 * the precision policy. Replaces ef::parse_efq (include/ef/qfile.h:133, src/qfile.cpp:125-223);
 * EFG_EFORMAT with the reference's message on the same faults. */
int efg_efq_check(const void* data, uint64_t size);

typedef struct {
  uint64_t file_bytes, bytes_per_token, source_tensor_bytes;
  int64_t override_extra_bytes; /* tensor bytes the overrides add versus the uniform policy */
  int32_t n_tensors;
  double seconds;
} efg_quantize_report;

/* Writes the .efq of a model directory (config.json + model.safetensors with BF16, F16 or
 * F32 tensors), quantizing on the GPU. Byte-identical to ef::quantize_model
 * (src/quantizer.cpp:151-290) for the same policy: `overrides` ("TENSOR=TYPE,...", or
 * "none"; ef::parse_overrides, src/qfile.cpp:94-115) when non-empty, else the named policy
 * `policy` ("auto", "uniform", "tinyllama-1.1b-chat-v1.0"; ef::select_policy,
 * src/quantizer.cpp:92-115). `report` may be NULL. EFG_EFORMAT for a checkpoint that does
 * not match its config, EFG_EINVAL for a bad policy or override. */
int efg_quantize_model(const char* model_dir, const char* out_file, const char* policy, const char* overrides,
                       efg_quantize_report* report);

typedef struct efg_decoder efg_decoder;

typedef struct {
  int32_t hidden, intermediate, layers, heads, kv_heads, head_dim, vocab, max_seq;
  int32_t n_q4, n_q8;       /* packed matrices of each type (embedding excluded) */
  int32_t embed_type;       /* EFG_* type of the token embedding */
  uint64_t bytes_per_token; /* weight bytes streamed per decoded token (src/qfile.cpp:237-241) */
} efg_model_info;

/* Loads an .efq (validated as efg_efq_check), uploads its data once to the current device,
 * allocates an FP32 KV cache of max_seq positions and records the decode step as CUDA
 * graphs. Replaces ef::Model::load_efq + the ef::Transformer constructor
 * (src/model.cpp:66-111, 153-182). Layer matrices and lm_head must be Q4_0 or Q8_0. */
int efg_decoder_open(const char* efq_path, size_t max_seq, efg_decoder** out);
int efg_decoder_close(efg_decoder* d);
int efg_decoder_info(const efg_decoder* d, efg_model_info* info);
/* ef::Transformer::reset (include/ef/model.h:102). */
int efg_decoder_reset(efg_decoder* d);
/* ef::Transformer::forward (src/model.cpp:184-276): runs `token` at `pos` (pos <= cached, a
 * smaller pos rewinds); writes the next-token logits to the host array `logits` (vocab
 * floats) unless it is NULL, which skips lm_head like compute_logits = false. */
int efg_decoder_forward(efg_decoder* d, int32_t token, size_t pos, float* logits);
/* The prompt as one batch: tokens[0..n) at positions pos0..pos0+n-1 (pos0 <= the cached
 * count), the same as n forward calls in turn (src/model.cpp:184-270), with the Q4_0
 * projections of all n tokens in one tensor-core GEMM per matrix instead of one matvec per
 * token (the reference prefills token by token, README.md:89-90). Writes the last token's
 * logits to `logits` (vocab floats) unless it is NULL. */
int efg_decoder_prefill(efg_decoder* d, const int32_t* tokens, size_t n, size_t pos0, float* logits);
/* ef::generate_greedy (src/model.cpp:278-304): prefill the prompt from position 0, then
 * argmax decoding of up to max_new tokens, stopping after eos_id (if >= 0). In the graph
 * mode the prompt goes through efg_decoder_prefill's batched path. With `forced`
 * (max_new ids) the decode steps are teacher-forced on those ids instead of the argmax,
 * while tokens_out still receives each step's argmax. step_logits (NULL or a host array of
 * (max_new - 1) * vocab floats) receives the logits after each decode forward. Times are
 * device time of the prefill and of the decode loop. */
int efg_decoder_generate(efg_decoder* d, const int32_t* prompt, size_t n_prompt, size_t max_new, int32_t eos_id,
                         const int32_t* forced, int32_t* tokens_out, size_t* n_tokens, float* step_logits,
                         double* prefill_seconds, double* decode_seconds);
/* Sequence slots for decoding several sequences together: slot 0 is the decoder's own KV
 * cache (forward, prefill, generate); slots 1..n_slots-1 get caches of their own, zeroed
 * (a second call resets them). */
int efg_decoder_set_slots(efg_decoder* d, size_t n_slots);
/* One decode step of n independent sequences at once (src/model.cpp:184-270 for each):
 * row b feeds tokens[b] at positions[b] (<= slot slots[b]'s cached count, which it rewinds
 * like forward) of slot slots[b] (distinct within a call). All rows share the weight
 * reads: Q4_0 projections as one tensor-core GEMM per matrix, Q8_0 ones one matvec per
 * row. Writes each row's logits (n * vocab floats) and its argmax (n ints) unless NULL.
 * No reference counterpart: the reference decodes one sequence at a time. */
int efg_decoder_step_slots(efg_decoder* d, const int32_t* slots, const int32_t* tokens, const int32_t* positions,
                           size_t n, float* logits, int32_t* next_tokens);
/* How the decode step runs: 0 = a CUDA graph of one kernel per operation (the default),
 * 1 = one persistent kernel per launch (one CTA per SM, the weights streamed through shared
 * memory across grid barriers). Both follow the reference's arithmetic. EFG_EINVAL when 1 is
 * asked for a model the persistent kernel cannot run. */
int efg_decoder_set_mode(efg_decoder* d, int persistent);
/* The current mode (0 or 1), -1 for a null handle. */
int efg_decoder_mode(const efg_decoder* d);

#ifdef __cplusplus
}
#endif
#endif /* EFG_H */
