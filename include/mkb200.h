/* C ABI of the B200 batch-one Qwen3-0.6B decode engine (libmkb200.so).
 *
 * Plain pointers and sizes only; every pointer named "device" is a CUDA device
 * pointer, every weight is BF16 in the reference's (Hugging Face nn.Linear)
 * [out, in] row-major layout unless stated. Weights and KV rows must be
 * 16-byte aligned (bulk-copy rule); a misaligned operand is reported as an error
 * instead of being copied.
 *
 * Error model: functions return cudaError_t. Launch-time errors come back
 * directly. In-kernel failures (a bounded wait that expired, bad arguments seen
 * on the device, a sum outside the fixed-point range) are
 *   - recorded in the workspace (read with mkb_workspace_status),
 *   - copied to an optional error word (mkb_decode_args.err_flag; the launchers
 *     point it at pinned host memory, so the host reads it without a copy),
 *   - made visible in the outputs: the failed launch writes NaN over its logits
 *     rows and -1 over every output token it did not complete.
 * A workspace that holds an error refuses further launches (outputs poisoned)
 * until it is reset. Launches on a library-owned workspace (launch_decode_kernel,
 * mkb_decode without a workspace, the engine calls) report an earlier
 * asynchronous launch's in-kernel failure the way CUDA reports asynchronous
 * errors: the next call returns cudaErrorLaunchFailure without launching, after
 * resetting the workspace; the call after it runs normally.
 */
#ifndef MKB200_H
#define MKB200_H

#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- drop-in for the reference launcher ------------------------------------
 * Same signature, argument meaning and return type as the reference's
 * `launch_decode_kernel` (megakernel.cu:898-927, declared in
 * pytorch_binding.cu:9-33). `layer_weights` is a DEVICE array of 28
 * LayerWeights structs (11 pointers each, config.cuh:77-89 order). Appends K/V
 * at `position`, attends over `cache_len` keys and writes FP32 logits to
 * `g_logits`. g_residual receives the final residual, g_q/g_k/g_v the last
 * layer's raw QKV projections and g_mlp_intermediate its SwiGLU vector;
 * hidden_buffer, g_activations, g_attn_output and g_normalized are not used.
 * The extra synchronisation workspace is allocated once per device on first use
 * (mkb_default_workspace); calls on one device must not overlap in time.
 * In-kernel failure: the logits are NaN, and the next launch on the device's
 * workspace returns cudaErrorLaunchFailure without launching (workspace reset).
 * The reference reported its errors through this return code alone. */
cudaError_t launch_decode_kernel(int token_id, const void* embed_weight, const void* lm_head_weight,
                                 const void* final_norm_weight, const void* layer_weights,
                                 const void* cos_table, const void* sin_table, void* k_cache, void* v_cache,
                                 void* hidden_buffer, void* g_residual, void* g_activations,
                                 void* g_attn_output, void* g_normalized, void* g_mlp_intermediate,
                                 void* g_logits, void* g_q, void* g_k, void* g_v, int position, int cache_len,
                                 int max_seq_len, cudaStream_t stream);

/* No counterpart in the reference. launch_decode_kernel with the same
 * arguments and results, for callers that must not allocate device memory at
 * any call: the synchronisation workspace lives in a file-scope device array of
 * at most 4 MiB per device (a build whose workspace is larger returns
 * cudaErrorInvalidValue). The first call on a device looks up that array's
 * address (cudaGetSymbolAddress) and caches it; make that first call before
 * any stream capture. Every call clears the workspace bytes with
 * cudaMemsetAsync on `stream`, then launches. The array is shared by all calls
 * on the device: calls that overlap in time race on it. An in-kernel failure
 * leaves NaN logits; its status stays readable with mkb_noalloc_status() after
 * the stream is synchronised and until the next call clears the array. */
cudaError_t launch_decode_kernel_noalloc(int token_id, const void* embed_weight, const void* lm_head_weight,
                                         const void* final_norm_weight, const void* layer_weights,
                                         const void* cos_table, const void* sin_table, void* k_cache,
                                         void* v_cache, void* hidden_buffer, void* g_residual,
                                         void* g_activations, void* g_attn_output, void* g_normalized,
                                         void* g_mlp_intermediate, void* g_logits, void* g_q, void* g_k,
                                         void* g_v, int position, int cache_len, int max_seq_len,
                                         cudaStream_t stream);
/* In-kernel status of launch_decode_kernel_noalloc's static workspace on
 * `device` (same words as mkb_workspace_status; synchronous copy, allocates
 * nothing). Read it after synchronising the launch's stream and before the next
 * launch_decode_kernel_noalloc call on that device, which clears it. */
cudaError_t mkb_noalloc_status(int device, uint32_t out[8]);

/* ---- explicit-argument launch ----------------------------------------------
 * Generalises the reference launcher (megakernel.cu:898-994): layer range,
 * input residual instead of the embedding gather, optional LM head, several
 * greedy tokens per launch, step state in device memory (for CUDA graphs), a
 * transposed down weight (fewer grid transitions) and FP32 RoPE tables. */
enum {
  MKB_FLAG_LM_HEAD = 1,          /* final norm + LM head + argmax */
  MKB_FLAG_SKIP_FINAL_NORM = 2,  /* LM head reads the residual as-is */
  MKB_FLAG_ADVANCE_STEP = 4      /* write argmax / position+1 back to `step` */
};

typedef struct mkb_decode_args {
  const void* embed;           /* device [vocab, 1024] */
  const void* lm_head;         /* device [vocab, 1024] (tied: == embed) */
  const void* final_norm;      /* device [1024] */
  const void* layers;          /* device LayerWeights[n_layers] */
  const void* down_t;          /* device array of n_layers pointers to [2][3072][512]
                                  transposed down weights (mkb_transpose_down), or NULL */
  const void* cos_table;       /* device [max_seq, 128] */
  const void* sin_table;
  int rope_fp32;               /* 1: FP32 tables, 0: BF16 */
  void* k_cache;               /* device [n_layers, 8, max_seq, 128] BF16 */
  void* v_cache;
  int max_seq;
  int layer_begin, layer_end;  /* run layers [begin, end) */
  int token, position, cache_len; /* used when step == NULL */
  int* step;                   /* device int[4] {token, position, -, count} or NULL */
  int n_tokens;                /* greedy tokens in this launch (>= 1) */
  int flags;
  const float* input_residual; /* device [1024] or NULL (embedding gather) */
  float* logits;               /* device [vocab] or NULL */
  int* out_tokens;             /* device [n_tokens] or NULL */
  float* residual_out;         /* device [1024] or NULL */
  float* q_out;                /* device [2048] / [1024] / [1024] / [3072] or NULL */
  float* k_out;                /*   (NULL: workspace scratch) */
  float* v_out;
  float* mlp_out;
  void* workspace;             /* device, mkb_workspace_bytes(); NULL = default */
  int grid;                    /* CTAs; 0 = one per SM */
  int splits;                  /* attention sequence splits; 0 = automatic */
  unsigned long long timeout_ns; /* bound on every in-kernel wait; 0 = 1 s */
  int withhold_cta;            /* test hook (-1 = off): that CTA never publishes its
                                  first QKV arrival, so the others' waits expire */
  unsigned long long* trace;   /* device [2*grid][trace_cap] time stamps or NULL; row c:
                                  consumers of CTA c, row grid+c: its producer. Record =
                                  (code << 48) | globaltimer_ns, code = kind | stage<<2 |
                                  layer<<7 | token<<12 (kind 0 wait begin, 1 wait end,
                                  2 publish, 3 mark; stage 0 QKV, 1 attention+o_proj,
                                  2 SwiGLU(+down), 3 down, 4 LM head, 5 split combine,
                                  6 token start, 7 token end, 8-15 sub-stage marks,
                                  16 ring slot fill wait, 17 producer slot wait,
                                  18 chunk issue) */
  int trace_cap;
  const int* prompt_tokens;    /* device int[n_tokens] or NULL: prefill mode. Token t of the
                                  launch is prompt_tokens[t] (not the previous argmax), and
                                  the LM head runs for the last token only. No counterpart
                                  in the reference (model.py:72-87 prefills with HF). */
  uint32_t* err_flag;          /* optional: receives the first in-kernel error code (device
                                  or mapped pinned host memory); NULL with workspace NULL
                                  = the device's own pinned word (checked by the next
                                  launch, see the error model above) */
  int stop_token;              /* -1 (default): none. Otherwise the launch ends after the
                                  first generated token equal to it (the reference loop's
                                  eos_token_id check, model.py:102-105): its id is the last
                                  one written, later out_tokens read -1, and no K/V row is
                                  appended for it. */
  int tp_rank, tp_size;        /* tensor parallel (no counterpart in the
                                  reference): tp_size 1 (default), 2, 4 or 8 GPUs, one
                                  launch per GPU at the same time. Rank r takes KV heads
                                  [r*8/tp_size, (r+1)*8/tp_size), SwiGLU rows and
                                  vocabulary rows in equal contiguous blocks; k_cache /
                                  v_cache are its [n_layers, 8/tp_size, max_seq, 128]
                                  shard; logits receives its vocabulary rows; the
                                  argmax is over the whole vocabulary. Needs down_t. */
  void* peer_workspaces[8];    /* tp_size > 1: every rank's workspace as this GPU
                                  addresses it (peer_workspaces[tp_rank] == workspace;
                                  the others mapped with mkb_ipc_open) */
  int* mailbox;                /* serve mode (with result): mapped pinned int[2] {seq, token};
                                  token t of the launch is taken once seq == t + 1 (a
                                  negative token ends the launch); NULL otherwise */
  int* result;                 /* serve mode: mapped pinned int[2] {seq, argmax}: the argmax
                                  of token t, then seq = t + 1 */
} mkb_decode_args;

void mkb_decode_args_init(mkb_decode_args* a);
cudaError_t mkb_decode(const mkb_decode_args* a, cudaStream_t stream);

/* ---- workspace ---------------------------------------------------------------- */
size_t mkb_workspace_bytes(void);
/* Zero a workspace (required after a launch reported an in-kernel error). */
cudaError_t mkb_workspace_reset(void* workspace, cudaStream_t stream);
/* Synchronous read of the in-kernel status: out[0] error code (0 = ok),
 * out[1] CTA, out[2] layer, out[3] stage, out[4] token. */
cudaError_t mkb_workspace_status(const void* workspace, uint32_t out[8]);
/* Read (and, when `set` is not NULL, first write) the workspace's tag base: the
 * tag of the last token decoded, from which tagged words are stamped. The
 * kernel restarts it at 0 (clearing every tagged word) once it passes 2^26;
 * writing it lets a test reach that point. Synchronous; no launch may be in
 * flight on the workspace. */
cudaError_t mkb_workspace_tag_base(void* workspace, const uint32_t* set, uint32_t* get);
/* The per-device workspace used when mkb_decode_args.workspace is NULL and by
 * launch_decode_kernel (allocated and zeroed on first use). */
cudaError_t mkb_default_workspace(int device, void** out);
const char* mkb_error_name(uint32_t code);

/* ---- layout helper -------------------------------------------------------------
 * down [1024, 3072] -> down_t [2][3072][512] (BF16): the transpose with its
 * 1024 output columns split into two contiguous 512-column blocks (one per CTA
 * of a cluster pair), the layout mkb_decode_args.down_t expects. */
cudaError_t mkb_transpose_down(const void* down, void* down_t, cudaStream_t stream);

/* ---- resident engine -------------------------------------------------------------
 * Keeps the device LayerWeights table, transposed down weights, workspace and a
 * CUDA graph of the per-token launch resident; the caller keeps ownership of
 * weights, RoPE tables and the KV cache. */
typedef struct mkb_model {
  const void* embed;
  const void* lm_head;
  const void* final_norm;
  const void* const* layer_weights; /* HOST array of n_layers*11 device pointers,
                                       LayerWeights order (model.py:30-44) */
  int n_layers;
  const void* cos_table;
  const void* sin_table;
  int rope_fp32;
  void* k_cache;
  void* v_cache;
  int max_seq;
  int fused_down;                   /* 1: transposed down weight (3 transitions/layer) */
  int use_graph;                    /* 1: replay the per-token launch as a CUDA graph */
  float* logits;                    /* device [vocab] for the last token's logits, or NULL
                                       (the engine then owns the buffer) */
  int tp_size;                      /* 0 or 1: one GPU. 2, 4, 8: one rank of a tensor-parallel
                                       group (k_cache/v_cache are the rank's 8/tp_size-head
                                       shard); every call is refused until mkb_engine_tp_attach */
} mkb_model;

typedef struct mkb_engine mkb_engine;
cudaError_t mkb_engine_create(const mkb_model* model, mkb_engine** out);
/* One token: host->device copy of (token, position), graph replay; the kernel
 * stores the argmax id straight into the engine's pinned (mapped) host memory.
 * Synchronises `stream`; the workspace status is read only when the token did
 * not complete. */
cudaError_t mkb_engine_step(mkb_engine* e, int token, int position, int* next_token, cudaStream_t stream);
/* n greedy tokens in one persistent launch, starting from `token` at `position`;
 * ids land in out_tokens (device, n entries). Asynchronous; a token that did not
 * complete reads -1, and the next engine call reports the failure
 * (cudaErrorLaunchFailure, workspace reset). */
cudaError_t mkb_engine_generate(mkb_engine* e, int token, int position, int n, int* out_tokens,
                                cudaStream_t stream);
/* As mkb_engine_generate, but the launch ends after the first generated token
 * equal to stop_token (>= 0; the reference loop stops on eos_token_id,
 * model.py:102-105): that id is the last one written, later entries read -1. */
cudaError_t mkb_engine_generate_until(mkb_engine* e, int token, int position, int n, int stop_token,
                                      int* out_tokens, cudaStream_t stream);
/* Serve session (no counterpart in the reference): one persistent launch that
 * decodes up to max_tokens tokens at positions position, position+1, ..., each
 * input token handed over by the host through pinned mapped memory and each
 * argmax handed back the same way, so a token costs no launch and no copy.
 * serve_open launches it on `stream` and returns; serve_step gives token t and
 * waits (host spin, bounded by timeout_ns) for its argmax; serve_close ends the
 * launch (after fewer than max_tokens steps too) and synchronises the stream.
 * Between steps the launch waits for the host at most timeout_ns (0 = 1 s),
 * then fails with a status. No other call may use the engine while a session is
 * open; TP engines are not supported. */
cudaError_t mkb_engine_serve_open(mkb_engine* e, int position, int max_tokens, unsigned long long timeout_ns,
                                  cudaStream_t stream);
cudaError_t mkb_engine_serve_step(mkb_engine* e, int token, int* next_token);
cudaError_t mkb_engine_serve_close(mkb_engine* e);
/* In-engine prefill: the n prompt ids (device int[n]) enter at positions
 * position .. position+n-1 in one persistent launch that appends their K/V rows;
 * the LM head runs for the last one only, whose argmax (the first generated
 * token) is written to *next_token (device int, may be NULL) and whose logits
 * stay in mkb_engine_logits(). Asynchronous. Replaces the HF prefill of
 * model.py:72-87 (no counterpart in the reference's kernel). */
cudaError_t mkb_engine_prefill(mkb_engine* e, const int* prompt_tokens, int n, int position, int* next_token,
                               cudaStream_t stream);
/* Batched prefill (no counterpart in the reference, which prefills with HF,
 * model.py:72-87): the n prompt ids (device int[n]) at positions position ..
 * position+n-1 go through each layer together -- projections as tcgen05
 * tensor-core GEMMs, causal attention on the tensor cores -- appending their
 * K/V rows; the last token's logits and greedy id are produced as by
 * mkb_engine_prefill. Asynchronous. Not for tensor-parallel engines. */
cudaError_t mkb_engine_prefill_batched(mkb_engine* e, const int* prompt_tokens, int n, int position, int* next_token,
                                      cudaStream_t stream);
/* The prefill's GEMM on its own: c[m, n] (FP32, row-major) = (a_hi + a_lo)[m, k]
 * b[n, k]^T with a_hi / a_lo / b BF16 row-major (16-byte aligned), n a multiple
 * of 128 (256-column tiles when n is a multiple of 256), k a multiple of 64.
 * Asynchronous. */
cudaError_t mkb_gemm_bf16_split(const void* a_hi, const void* a_lo, const void* b, float* c, int m, int n, int k,
                                cudaStream_t stream);
float* mkb_engine_logits(mkb_engine* e);   /* device [vocab], last token's logits */
void* mkb_engine_workspace(mkb_engine* e);
/* Tensor parallel: make this rank's engine one of tp_size (2, 4 or 8) engines
 * that decode together, one per GPU, every call made on every rank with the
 * same arguments. peer_workspaces[g] is rank g's mkb_engine_workspace() as this
 * GPU addresses it (its own for g == tp_rank; the others through
 * mkb_ipc_export / mkb_ipc_open). The engine's KV cache must be the rank's
 * [n_layers, 8/tp_size, max_seq, 128] shard and it must use the transposed down
 * weight. Re-captures the step graph. No counterpart in the reference. */
cudaError_t mkb_engine_tp_attach(mkb_engine* e, int tp_rank, int tp_size, void* const* peer_workspaces);
/* Device memory shared across processes for the peer workspaces (CUDA IPC):
 * export writes 64 opaque bytes for a cudaMalloc'd pointer; open maps another
 * process's exported pointer into this one (NVLink peer access); close unmaps. */
cudaError_t mkb_ipc_export(const void* device_ptr, unsigned char handle[64]);
cudaError_t mkb_ipc_open(const unsigned char handle[64], void** device_ptr);
cudaError_t mkb_ipc_close(void* device_ptr);
int mkb_engine_grid(mkb_engine* e);
void mkb_engine_destroy(mkb_engine* e);

/* ---- schedule introspection (host only, no GPU needed) ------------------------ */
/* out[0..13] = qa, qb, in_bc, h, c, oa, ob, ja, jb, da, db, va, vb, group_size. */
int mkb_plan_query(int grid, int cta, int32_t out[16]);
/* The same for rank tp_rank of a tp_size-GPU launch; out[14] = the CTA's local
 * KV head (cache shard index); qa/qb are in the rank's local QKV row space,
 * mapped to [Wq; Wk; Wv] rows by mkb_qkv_global_row. */
int mkb_plan_query_tp(int grid, int cta, int tp_rank, int tp_size, int32_t out[16]);
int mkb_qkv_global_row(int tp_rank, int tp_size, int local_row);
/* Attention splits the kernel uses for a token at this cache length (when
 * mkb_decode_args.splits is 0): 1 below 385 keys, else one split per 64-key
 * chunk, at most group_size. */
int mkb_choose_splits(int cache_len, int group_size);
void mkb_key_range(int cache_len, int splits, int c, int32_t out[2]);
/* Keys [out[0], out[1]) that CTA `cta` of a `grid`-CTA launch attends over at
 * this cache length (split across the head group, or halved between the two
 * CTAs of a cluster pair that share the KV head); returns whether the pair
 * shares its head. */
int mkb_attn_keys(int cache_len, int splits, int grid, int cta, int32_t out[2]);
int mkb_qkv_chunk_end(int r, int qb);
size_t mkb_smem_bytes(void);
int mkb_version(void);

#ifdef __cplusplus
}
#endif

#endif /* MKB200_H */
