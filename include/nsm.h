/*
 * nsm.h -- C ABI of the B200-native blockwise-sparse NF4 decode MLP.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t,
 * returns an int status (NSM_OK == 0, negative on error), never throws,
 * never allocates device memory, and is ordered on the given stream.  Scratch
 * memory is a caller-owned workspace whose size is returned by the matching
 * *_workspace_bytes() query; its address must be 256-byte aligned (as every
 * CUDA allocation is), else the call returns NSM_ERR_WORKSPACE.  A workspace
 * must be zero-filled once before its first use (nsm_workspace_init); every
 * call leaves its counters zero again.  Calls that share one workspace must not overlap on the GPU.
 *
 * The reference (andott28/next_step_ai) has no native code: its hot path is
 * Python + Triton.  Each declaration below names the reference interface it
 * replaces (paths relative to the reference checkout).
 *
 * NF4 conventions (as in the reference): element e of a row-major weight lives
 * in byte e/2, high nibble = even element; value = code[nibble] *
 * absmax[e / quant_block_size].  This build's fast paths require
 * block_size == 32 and quant_block_size == 64 (the configuration the
 * reference's single-kernel path requires, triton_sparse_mlp.py:1401-1406).
 */
#ifndef NSM_H_
#define NSM_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* nsm_stream_t; /* == cudaStream_t */

/* ---- status codes ---------------------------------------------------- */
#define NSM_OK 0
#define NSM_ERR_INVALID_ARG (-1)   /* bad pointer / size / layout         */
#define NSM_ERR_UNSUPPORTED (-2)   /* shape outside the supported set     */
#define NSM_ERR_CUDA (-3)          /* a CUDA runtime call failed          */
#define NSM_ERR_TIMEOUT (-4)       /* a bounded device wait gave up       */
#define NSM_ERR_WORKSPACE (-5)     /* workspace missing, misaligned or too small */
#define NSM_ERR_DEVICE (-6)        /* device is not sm_100 / not present  */

/* ---- element types --------------------------------------------------- */
#define NSM_F32 0
#define NSM_F16 1
#define NSM_BF16 2

int nsm_abi_version(void);
const char* nsm_status_string(int status);
/* Detail of the last failing call on the calling host thread. */
const char* nsm_last_error(void);
/* Zero-fills a workspace (stream-ordered). */
int nsm_workspace_init(void* ws, size_t ws_bytes, nsm_stream_t stream);
/* Reads (and clears) the workspace's device error word: kernels that give up
 * on a bounded wait record a status there (NSM_ERR_TIMEOUT) instead of
 * spinning.  Synchronises `stream`.  *code_out = 0 when no kernel failed. */
int nsm_workspace_error(void* ws, size_t ws_bytes, int32_t* code_out, nsm_stream_t stream);

/* ---- router ------------------------------------------------------------
 * Learned-basis router weights.  Replaces the per-layer routing dict the
 * reference builds at streaming_llama_runtime.py:849-991 and consumes in
 * _compute_sparse_basis_latent / _route_sparse_mlp (:4209-4238, :4311-4352).
 *   enc_w   [rank, H]    enc_b [rank] (may be NULL)
 *   score_w [NB, rank]   score_b [NB] (may be NULL)       -- learned head
 *   legacy_abs_latent=1: scores = |latent| @ score_w^T with score_w = dec_norm_t^T
 *   down_block_norm [NB] fp32 (may be NULL): scores *= down_block_norm
 * weight_dtype applies to enc_w, enc_b, score_w, score_b.                 */
typedef struct nsm_router_weights {
  const void* enc_w;
  const void* enc_b;
  const void* score_w;
  const void* score_b;
  const float* down_block_norm;
  int32_t weight_dtype;
  int32_t rank;
  int32_t num_blocks;
  int32_t top_k;
  int32_t basis_top_k;
  int32_t legacy_abs_latent;
} nsm_router_weights;

/* ---- NF4 MLP weights ---------------------------------------------------
 * Replaces the gathered / hot-pool tensors the reference passes to
 * _sparse_mlp_forward_fast_triton (streaming_llama_runtime.py:5526-5547)
 * and to triton_sparse_mlp_decode_4bit_single_kernel_sm75
 * (triton_sparse_mlp.py:1378-1396).
 *
 * gate/up: one 32-row block per "pool row", bitsandbytes row-major inside a
 *   block: byte (row i, col c) of pool row p at
 *   gate_packed + p*gateup_block_stride + i*(H/2) + c/2; fp32 absmax at
 *   gate_absmax + p*gateup_absmax_block_stride + i*(H/64) + c/64.
 *   Strides 0 mean the dense values 16*H and H/2.
 * down: the 16 packed bytes of row h of pool row p at
 *   down_packed + p*down_block_stride + h*down_row_stride; its absmax at
 *   down_absmax[p*down_absmax_block_stride + h*down_absmax_row_stride].
 *   Block-major [P][H][16] + [P][H]: strides (16*H, 16, H, 1) (the default
 *   when all four are 0).  The reference's gathered columns [H][U][16] +
 *   [H][U]: (16, 16*U, 1, U).  A whole bitsandbytes down weight [H][I/2] +
 *   [H][I/64] addressed by block id: (16, I/2, 1, I/64) with
 *   down_absmax_pair=1.
 * down_absmax_pair=1 means the absmax index of block b is b/2 (64-column
 *   quant groups over 32-column blocks), as in the reference's column
 *   gather abs_idx = (b*32)//64 (streaming_llama_runtime.py:4510).       */
typedef struct nsm_mlp_weights {
  const uint8_t* gate_packed;
  const float* gate_absmax;
  const uint8_t* up_packed;
  const float* up_absmax;
  const uint8_t* down_packed;
  const float* down_absmax;
  const float* gate_code; /* [16] fp32 */
  const float* up_code;
  const float* down_code;
  const void* gate_bias;  /* [I] (indexed by block*32+row) or NULL */
  const void* up_bias;
  const void* down_bias;  /* [H] or NULL */
  int32_t bias_dtype;
  int32_t pool_rows;      /* number of valid pool rows                   */
  int64_t gateup_block_stride;
  int64_t gateup_absmax_block_stride;
  int64_t down_block_stride;
  int64_t down_row_stride;
  int64_t down_absmax_block_stride;
  int64_t down_absmax_row_stride;
  int32_t down_absmax_pair;
  int32_t layout;         /* NSM_LAYOUT_* bits */
} nsm_mlp_weights;

/* nsm_mlp_weights.layout bits.  Without them gate/up and down use the
 * bitsandbytes / strided layouts above.  With them a pool row holds the
 * lane-interleaved "tiled" layout written by nsm_repack_tiled (same bytes
 * per block: gate/up 16*H packed + H/2 absmax floats, down 16*H + H):
 *   gate/up packed: [H/64 column tiles][2 row groups][32 lanes][16 B], lane
 *     (g=lane/4, t=lane%4) holding bytes [8t, 8t+8) of the tile in rows
 *     16*rg+g and 16*rg+g+8;
 *   gate/up absmax: [H/64 tiles][8 g][4] = rows g, g+8, 16+g, 24+g;
 *   down packed: [H/32 row tiles][32 lanes][16 B], lane (g,t) holding bytes
 *     [4t, 4t+4) of rows g, g+8, 16+g, 24+g of the tile;
 *   down absmax: [H/32 row tiles][8 g][4] (same four rows).
 * Block strides are unchanged; the row strides of the strided layouts are
 * ignored for a tiled part. */
#define NSM_LAYOUT_GATEUP_TILED 1
#define NSM_LAYOUT_DOWN_TILED 2
/* gate_code and up_code hold the same 16 values (the standard NF4 codebook
 * does).  The tiled gate/up kernel then serves both projections from one
 * lookup table and runs more warps in the shared memory that frees; it
 * checks the claim and records NSM_ERR_INVALID_ARG in the workspace error
 * word (computing nothing) when the codebooks differ. */
#define NSM_LAYOUT_SHARED_CODE 4

/* Block -> pool-row mapping applied to the router's selection.
 *   slot_of_block [NB] int32 (device): pool row, or <0 = not present here.
 *   If NULL: pool row = block - block_begin for block_begin <= block < block_end,
 *   other blocks are not present here (multi-GPU shards; [0,NB) = everything). */
typedef struct nsm_block_map {
  const int32_t* slot_of_block;
  int32_t block_begin;
  int32_t block_end;
} nsm_block_map;

/* Residual / RMSNorm prologue of a decoder layer (optional).
 *   If residual != NULL: residual[H] (fp32, in/out) += y_prev[H] (if not NULL,
 *   y_prev_dtype) and the MLP input is rmsnorm(residual) * norm_weight, as the
 *   reference's post_attention_layernorm + residual add
 *   (streaming_llama_runtime.py:7762-7775).  Otherwise x is the MLP input. */
typedef struct nsm_layer_io {
  float* residual;
  const void* y_prev;
  int32_t y_prev_dtype;
  int32_t norm_weight_dtype;
  const void* norm_weight; /* [H] or NULL (= ones) */
  float eps;
  /* flags: NSM_IO_PENDING_Y -- instead of y_prev, the previous layer's output
   *   is still pending in this workspace as down-projection partials (from a
   *   call with NSM_IO_DEFER_Y on the same workspace); they are summed here in
   *   fixed order (and across ranks through `exchange`) before the residual add.
   * NSM_IO_DEFER_Y -- leave this layer's output pending in the workspace
   *   instead of writing y (y may be NULL); the next layer (NSM_IO_PENDING_Y)
   *   or nsm_residual_flush consumes it.  Needs a down projection without bias. */
  int32_t flags;
  int32_t reserved2;
  /* Cross-GPU sum of the pending output (NULL on one GPU): every rank's
   * partial is pushed to every rank over NVLink and summed in rank order inside
   * the router's first kernel -- the all-reduce of the reference configuration
   * fused with the residual add. */
  const struct nsm_exchange* exchange;
  /* Optional timing hook: NSM_STAGE_EVENTS cudaEvent_t handles recorded on the
   * stream before the router, before gate/up, before the gate/up reduction,
   * before down, before the down reduction and after it.  Recording them
   * separates the kernels (no programmatic dependent launch across a stage
   * boundary), so use it for per-kernel timing only.  NULL: no events. */
  void* const* stage_events;
} nsm_layer_io;
#define NSM_STAGE_EVENTS 6
#define NSM_IO_PENDING_Y 1
#define NSM_IO_DEFER_Y 2

/* residual += the pending output of the last NSM_IO_DEFER_Y layer (summed
 * across ranks through io->exchange when set).  io->residual is required;
 * io->flags must include NSM_IO_PENDING_Y. */
int nsm_residual_flush(int32_t hidden, const nsm_layer_io* io, void* ws, size_t ws_bytes, nsm_stream_t stream);

/* ---- cross-GPU exchange buffers --------------------------------------------
 * One per rank (one process per GPU of a node).  nsm_exchange_create
 * allocates this rank's buffer (cudaMalloc, zeroed; the only allocating calls
 * of this library besides nothing else) and writes its CUDA IPC handle
 * (NSM_IPC_HANDLE_BYTES bytes) for the other ranks; nsm_exchange_connect
 * opens the peers' buffers from all ranks' handles (world x
 * NSM_IPC_HANDLE_BYTES, in rank order).  No counterpart in the reference (it
 * is single-GPU); replaces the NCCL all-reduce of the multi-GPU configuration. */
#define NSM_IPC_HANDLE_BYTES 64
typedef struct nsm_exchange nsm_exchange;
size_t nsm_exchange_bytes(int world, int hidden);
int nsm_exchange_create(int32_t world, int32_t rank, int32_t hidden, nsm_exchange** ex_out, void* ipc_handle_out);
int nsm_exchange_connect(nsm_exchange* ex, const void* handles);
int nsm_exchange_destroy(nsm_exchange* ex);
/* Connects n exchanges created in ONE process (ranks 0..n-1 of one world,
 * in rank order) to each other directly, without IPC handles: for one process
 * driving several ranks whose buffers every rank's device can reach (the
 * caller enables peer access between different devices).  Kernels of ranks
 * that wait on each other must never run as separate launches on one GPU;
 * a single-GPU caller only launches one rank (the tests use it to make a wait
 * run out).  No counterpart in the reference. */
int nsm_exchange_connect_local(nsm_exchange* const* exs, int32_t n);
/* Polls of one peer word the router makes before it gives up on a rank that
 * never delivered and records NSM_ERR_TIMEOUT in the workspace error word
 * (nsm_workspace_error) -- the bounded wait of the fused exchange.  0 = the
 * default (2^24 polls, seconds).  Applies to launches issued after the call
 * (a captured graph keeps the value it was captured with).  No counterpart in
 * the reference (its runtime is single-GPU). */
int nsm_exchange_set_spin_limit(nsm_exchange* ex, int32_t spins);

size_t nsm_decode_workspace_bytes(int hidden, int intermediate, int top_k, int rank);
/* Process-wide bound on a warp's wait for its own bulk copies (mbarrier tries)
 * in the gather-GEMV kernels; a wait that runs out records NSM_ERR_TIMEOUT in
 * the workspace error word, drains the warp's copies in flight and stops the
 * warp.  0 = the default (2^22 tries).  Returns the previous bound (or a
 * negative status for a negative argument).  Applies to later launches.  No
 * counterpart in the reference. */
int nsm_set_copy_wait_limit(int32_t spins);
/* The blocks the last nsm_sparse_mlp_decode on this workspace computed (the
 * router's selection present in the pool, ascending block ids) and their
 * count: copies the workspace's selection record to blocks_out [min(top_k,
 * intermediate/32)] and count_out [1] (both device int32; stream-ordered).
 * hidden, intermediate, top_k and rank are the values that call used.  The
 * selection the decode path makes inside its gate/up kernel (no idx_out) is
 * otherwise never returned; this exposes the rows the reference's
 * _route_sparse_mlp result would give (streaming_llama_runtime.py:4311-4352,
 * sorted by block id as _build_sparse_active_layout orders them, :4857-4908). */
int nsm_workspace_selection(const void* ws, size_t ws_bytes, int32_t hidden, int32_t intermediate, int32_t top_k,
                            int32_t rank, int32_t* blocks_out, int32_t* count_out, nsm_stream_t stream);

/* Router only (latent GEMV + block scores + top-k), one token.
 * Replaces StreamingLlamaRuntime._route_sparse_mlp for rows == 1
 * (streaming_llama_runtime.py:4311-4352).  idx_out [top_k] int32 block ids in
 * score-descending order (ties: lower block id first); score_out [top_k]
 * fp32 (may be NULL); latent_out [rank] fp32 (may be NULL). */
int nsm_route(const void* x, int32_t x_dtype, int32_t hidden, const nsm_router_weights* rw,
              int32_t* idx_out, float* score_out, float* latent_out, void* ws, size_t ws_bytes,
              nsm_stream_t stream);

/* Router for `rows` tokens at once: x [rows][hidden] row-major; idx_out
 * [rows][top_k], score_out [rows][top_k] (may be NULL), latent_out
 * [rows][rank] (may be NULL), each row as nsm_route would give it.  Replaces
 * StreamingLlamaRuntime._route_sparse_mlp for rows > 1
 * (streaming_llama_runtime.py:4311-4352): three launches for all rows.
 * Workspace: nsm_route_workspace_bytes(hidden, num_blocks, top_k, rank, rows). */
size_t nsm_route_workspace_bytes(int hidden, int num_blocks, int top_k, int rank, int rows);
int nsm_route_rows(const void* x, int32_t x_dtype, int32_t rows, int32_t hidden, const nsm_router_weights* rw,
                   int32_t* idx_out, float* score_out, float* latent_out, void* ws, size_t ws_bytes,
                   nsm_stream_t stream);

/* Whole decode MLP for one token: route, gather-GEMV gate/up, SiLU*up,
 * gather-GEMV down.  Replaces _mlp_forward_dispatch's decode branch
 * (streaming_llama_runtime.py:5906-5913) = _route_sparse_mlp +
 * _sparse_mlp_forward_fast (:5104) with resident blocks.
 *   x [H] (x_dtype) unless io.residual is set (then x is ignored).
 *   idx_in: if not NULL, [k_in] int32 block ids replace the router (rw may
 *   then be NULL).  y [H] in y_dtype: the MLP output (the partial over the
 *   blocks present here when the map selects a shard).
 *   idx_out/score_out (may be NULL): the router's selection. */
int nsm_sparse_mlp_decode(const void* x, int32_t x_dtype, int32_t hidden, int32_t intermediate,
                          const nsm_layer_io* io, const nsm_router_weights* rw, const int32_t* idx_in,
                          int32_t k_in, const nsm_block_map* map, const nsm_mlp_weights* w, void* y,
                          int32_t y_dtype, int32_t* idx_out, float* score_out, void* ws, size_t ws_bytes,
                          nsm_stream_t stream);

/* Decode MLP on blocks the caller already gathered, in the reference
 * runtime's layout: gate/up [U][32][H/2] + [U][32][H/64], down [H][U][16] +
 * [H][U].  Replaces triton_sparse_mlp_decode_4bit_single_kernel_sm75
 * (triton_sparse_mlp.py:1378-1516) and the rows == 1 use of
 * _sparse_mlp_forward_fast_triton (streaming_llama_runtime.py:5579-5625);
 * unlike the reference it is not restricted to sm_75.
 *   act_out [U*32] fp32 (may be NULL): SiLU(gate)*up. */
int nsm_decode_gathered(const void* x, int32_t x_dtype, int32_t hidden, int32_t num_blocks_gathered,
                        const nsm_mlp_weights* w, void* y, int32_t y_dtype, float* act_out, void* ws,
                        size_t ws_bytes, nsm_stream_t stream);

/* Multi-row decode on gathered blocks with the reference's per-row mask:
 * y[r] = down(silu(gate(x[r]) * flat_mask[r]) * (up(x[r]) * flat_mask[r])).
 * Replaces the rows > 1 branch of _sparse_mlp_forward_fast
 * (streaming_llama_runtime.py:5433-5492, layout from :4857-4908).
 *   x [rows][H]; flat_mask [rows][U*32] (mask_dtype); y [rows][H]. */
size_t nsm_decode_rows_workspace_bytes(int hidden, int num_blocks_gathered, int rows);
int nsm_decode_gathered_rows(const void* x, int32_t x_dtype, int32_t rows, int32_t hidden,
                             int32_t num_blocks_gathered, const void* flat_mask, int32_t mask_dtype,
                             const nsm_mlp_weights* w, void* y, int32_t y_dtype, void* ws, size_t ws_bytes,
                             nsm_stream_t stream);

/* nsm_decode_gathered without a workspace argument, for callers that cannot
 * allocate device memory when they decode (a fixed pool sized before serving
 * starts, a binding with no access to the CUDA allocator).  It has no
 * counterpart in the reference.  It allocates nothing: its scratch is a
 * 6.5 MiB array inside the library that each device using it holds until the
 * process exits.  Limits: hidden <= NSM_STATIC_MAX_HIDDEN, num_blocks_gathered
 * <= NSM_STATIC_MAX_BLOCKS; larger calls return NSM_ERR_UNSUPPORTED.  All
 * calls on a device share the array (each clears what must start at zero), so
 * calls that overlap on the GPU race.  The first call on a device sets up the
 * array's address with that device current; make it before any stream
 * capture.  Results equal nsm_decode_gathered's. */
#define NSM_STATIC_MAX_HIDDEN 16384
#define NSM_STATIC_MAX_BLOCKS 256
int nsm_decode_gathered_static(const void* x, int32_t x_dtype, int32_t hidden, int32_t num_blocks_gathered,
                               const nsm_mlp_weights* w, void* y, int32_t y_dtype, float* act_out,
                               nsm_stream_t stream);
/* The device error word of nsm_decode_gathered_static's array on the current
 * device: *code_out = NSM_ERR_TIMEOUT when a kernel of an earlier static call
 * gave up on a bounded wait (its output is then incomplete), else 0; the word
 * is cleared.  Synchronises `stream`; allocates nothing.  The calls do not
 * clear the word themselves, so one check after several calls covers them
 * all.  Like the entry point it serves, no counterpart in the reference. */
int nsm_static_error(int32_t* code_out, nsm_stream_t stream);

/* ---- one token through a whole layer stack, one kernel ------------------
 * The per-token layer loop of the reference's decode
 * (StreamingLlamaRuntime.forward_token, streaming_llama_runtime.py:7612-7775)
 * restricted to the MLP path -- for every layer: residual += the previous
 * layer's MLP output, x = rmsnorm(residual) * norm_weight, _route_sparse_mlp
 * (:4311-4352), the exact blockwise-sparse MLP on the selected blocks
 * (:5433-5492) -- with attention left out (identity), run as ONE persistent
 * cooperative kernel: the phases of a layer are linked inside the kernel by
 * bounded waits on arrival counters, so a token costs one launch.
 * Requirements: router rank 64, bf16 or fp16 router weights, top_k <= 256,
 * at most 4096 blocks, hidden a multiple of 128 and at most 16384, tiled pools
 * (NSM_LAYOUT_GATEUP_TILED | NSM_LAYOUT_DOWN_TILED), no biases, 16-byte
 * aligned pools and strides, and a down codebook equal (by value) to the gate
 * or the up codebook (a kernel that finds otherwise records
 * NSM_ERR_UNSUPPORTED in the workspace error word).
 * Numerics: x and SiLU(gate)*up enter the tensor cores as fp16 hi + lo pairs,
 * the codebooks as fp16(alpha * code) with a per-codebook alpha in [1, 2)
 * that minimises their fp16 rounding (1/alpha applied in fp32 with the
 * absmax); accumulation is fp32. */
typedef struct nsm_token_layer {
  nsm_router_weights router;
  nsm_mlp_weights mlp;
  nsm_block_map map;          /* the blocks this rank's pools hold */
  const void* norm_weight;    /* [H] RMSNorm weight of the MLP input, or NULL */
  int32_t norm_weight_dtype;
  int32_t reserved;
} nsm_token_layer;
/* Workspace of nsm_decode_token for num_layers layers; zero-fill it once
 * (nsm_workspace_init).  Its error word is read by nsm_workspace_error. */
size_t nsm_token_workspace_bytes(int hidden, int intermediate, int num_layers);
/* Validates the layers and copies their descriptors into the workspace
 * (synchronises `stream`; not capturable).  The weights must stay valid while
 * the workspace is used. */
int nsm_token_set_layers(void* ws, size_t ws_bytes, int32_t hidden, int32_t intermediate,
                         const nsm_token_layer* layers, int32_t num_layers, nsm_stream_t stream);
/* One token through the num_layers layers set on the workspace: residual [H]
 * fp32 (in/out) ends as residual + every layer's MLP output.  ex: the cross-GPU
 * exchange when the blocks are sharded over ranks (NULL on one GPU).  Optional
 * records for tests (NULL to skip): trace_blocks [num_layers][trace_k] the
 * selected blocks present here, ascending; trace_counts [num_layers];
 * trace_residual [num_layers][H] the residual each layer's RMSNorm read.
 * Calls sharing a workspace must not overlap on the GPU. */
int nsm_decode_token(float* residual, int32_t hidden, int32_t intermediate, int32_t num_layers, float eps,
                     const nsm_exchange* ex, int32_t* trace_blocks, int32_t trace_k, int32_t* trace_counts,
                     float* trace_residual, void* ws, size_t ws_bytes, nsm_stream_t stream);
/* Profiling hook of nsm_decode_token: with stamps != NULL, later calls on this
 * workspace write 8 globaltimer readings (ns) per CTA for each of the first
 * stamp_layers layers -- stamps[(layer * ctas + cta) * 8 + i], i = phase A
 * start, A done, B start, B done, selection done, gate/up done, activations
 * ready, down done (ctas = the SM count) -- for reading where a token's time
 * goes.  stamps == NULL switches it off.  Synchronises `stream`. */
int nsm_token_profile(void* ws, size_t ws_bytes, int32_t hidden, int32_t intermediate, int32_t num_layers,
                      unsigned long long* stamps, int32_t stamp_layers, nsm_stream_t stream);

/* ---- multi-token decode over the union of the tokens' blocks ------------
 * Up to 32 tokens: x [rows][H] (x_dtype), idx [rows][k] int32 block ids (each
 * row's router selection; ids < 0 or >= NB are ignored), the resident pools
 * (tiled gate/up and down layouts, no biases) and block map -> y [rows][H]
 * (y_dtype).  The union of the rows' blocks present in the pool is formed in
 * ascending block order with one row mask per union block -- the reference's
 * _build_sparse_active_layout (streaming_llama_runtime.py:4857-4908) -- and
 * each union block's NF4 tiles are dequantised once and multiplied against all
 * rows on the tensor cores; row r's SiLU(g)*u is zero outside its own blocks
 * (the reference's flat_mask, :5451-5492).
 *   union_out [min(NB, rows*k)] (may be NULL): the union's block ids;
 *   union_count_out (device int32, may be NULL): its size. */
size_t nsm_union_workspace_bytes(int hidden, int intermediate, int rows, int k);
int nsm_union_decode(const void* x, int32_t x_dtype, int32_t rows, int32_t hidden, int32_t intermediate,
                     const int32_t* idx, int32_t k, const nsm_block_map* map, const nsm_mlp_weights* w, void* y,
                     int32_t y_dtype, int32_t* union_out, int32_t* union_count_out, void* ws, size_t ws_bytes,
                     nsm_stream_t stream);

/* ---- layout helpers ----------------------------------------------------- */
/* bitsandbytes down weight [H][I/2] + absmax [H][I/64] -> block-major
 * [n][H][16] + [n][H] for the listed blocks (blocks == NULL: all I/32).
 * Replaces the column extraction of _load_down_proj_cold_cols /
 * _maybe_cache_down_proj_hot_columns (streaming_llama_runtime.py:4497-4513,
 * :2664-2674). */
int nsm_repack_down_block_major(const uint8_t* down_packed, const float* down_absmax, int32_t hidden,
                                int32_t intermediate, const int32_t* blocks, int32_t n, uint8_t* out_packed,
                                float* out_absmax, nsm_stream_t stream);

/* bitsandbytes row-major NF4 weights -> tiled pool rows (layout above).
 *   gate/up: [n_src][32][H/2] + [n_src][32][H/64] (block b at b*16H bytes);
 *   down: the whole [H][I/2] + [H][I/64] weight, blocks picked by id.
 * Block blocks[i] (all blocks when blocks == NULL) goes to destination row
 * i (dst_rows == NULL) or dst_rows[i]; dst pointers/strides come from `dst`
 * (its layout bits are ignored).  Either source may be NULL to skip it. */
int nsm_repack_tiled(const uint8_t* gate_packed, const float* gate_absmax, const uint8_t* up_packed,
                     const float* up_absmax, const uint8_t* down_packed, const float* down_absmax, int32_t hidden,
                     int32_t intermediate, const int32_t* blocks, const int32_t* dst_rows, int32_t n,
                     const nsm_mlp_weights* dst, nsm_stream_t stream);

/* ---- reference Triton API semantics --------------------------------------
 * triton_sparse_input_linear_4bit (triton_sparse_mlp.py:1303-1337, kernels
 * :437-575): out[r][n] = bias[n] + sum over slots of active_idx[r] >= 0 and
 * i < block_size of W(e=(blk*bs+i)*out_features+n) * x[r][blk*bs+i].
 * x, bias, out in act_dtype; accumulation fp32. */
int nsm_sparse_input_linear_4bit(const void* x, int32_t act_dtype, int32_t rows, const int32_t* active_idx,
                                 int32_t top_k, const uint8_t* packed, const float* absmax, const float* code,
                                 int32_t out_features, int32_t in_features, int32_t quant_block_size,
                                 const void* bias, int32_t block_size, void* out, nsm_stream_t stream);

/* triton_sparse_output_linear_4bit (triton_sparse_mlp.py:1340-1375, kernel
 * :578-651): out[r][blk*bs+o] = (bias[blk*bs+o] + sum_k W(e=k*bs+blk*bs+o) *
 * x[r][k]) * flat_mask[r][blk*bs+o]; other columns 0.  out is [rows][width]. */
int nsm_sparse_output_linear_4bit(const void* x, int32_t act_dtype, int32_t rows, const int32_t* active_idx,
                                  int32_t top_k, const void* flat_mask, int32_t width, const uint8_t* packed,
                                  const float* absmax, const float* code, int32_t input_dim,
                                  int32_t quant_block_size, const void* bias, int32_t block_size, void* out,
                                  nsm_stream_t stream);

/* ---- VRAM hot-block cache ------------------------------------------------
 * Device side of the reference's hot-block cache
 * (streaming_llama_runtime.py:2619-2786, :2809-3018).  The policy
 * (_plan_fixed_capacity_bank_update, :2577-2617) runs on the host; these
 * move bytes and tables.
 * nsm_cache_split: for idx[k] and slot_of_block[NB], writes hit_rows[] (pool
 * rows of resident blocks, in idx order), miss_pos[] (positions in idx of
 * the misses) and counts[2] = {hits, misses} (all device). */
int nsm_cache_split(const int32_t* idx, int32_t k, const int32_t* slot_of_block, int32_t num_blocks,
                    int32_t* hit_rows, int32_t* miss_pos, int32_t* counts, nsm_stream_t stream);

/* Copies pool rows src_rows[i] -> dst_rows[i] (gate, up, down and absmax of
 * each block) inside the same pools and sets slot_of_block[block_ids[i]] =
 * dst_rows[i], slot_of_block[evicted_ids[i]] = -1 when evicted_ids[i] >= 0.
 * Replaces the promotion copies of _promote_down_proj_hot_columns_from_gpu
 * (:2995-3003) and _promote_sparse_param_hot_blocks_from_gpu (:2872-2877). */
int nsm_cache_promote(const nsm_mlp_weights* w, int32_t hidden, const int32_t* src_rows, const int32_t* dst_rows,
                      const int32_t* block_ids, const int32_t* evicted_ids, int32_t n, int32_t* slot_of_block,
                      nsm_stream_t stream);

/* Stages blocks from a host block store of host_records records into device
 * pool rows: block blocks[i] (record host_base + blocks[i]*record_bytes) ->
 * pool row dst_rows[i] (pool_base + dst_rows[i]*record_bytes), on `stream` (a
 * side stream, so the copies overlap the resident-block compute).  When
 * host_base is pinned host memory the device can address (cudaHostAlloc /
 * pinned torch tensors) and the records are 16-byte multiples, one gather
 * kernel reads all records over the host link; otherwise one cudaMemcpyAsync
 * per block.  blocks and dst_rows are HOST arrays, checked against
 * host_records and pool_rows before anything is queued.  A record holds all
 * of one block's bytes (gate, up, down and their absmax).  Replaces the
 * pinned host-to-device copies of _copy_cpu_to_gpu and the cold block loads
 * (streaming_llama_runtime.py:3443-3493, :3885-4002). */
int nsm_cache_stage(const void* host_base, int32_t host_records, const int32_t* blocks, int32_t n,
                    size_t record_bytes, void* pool_base, const int32_t* dst_rows, int32_t pool_rows,
                    nsm_stream_t stream);

/* ---- NF4 LM head ---------------------------------------------------------
 * logits[t][v] = sum_h code[nib(v*H+h)] * absmax[(v*H+h)/qbs] * x[t][h] (+ bias[v])
 * for a bitsandbytes row-major NF4 weight W [V = out_features, H = in_features]
 * (flat bytes, element e in byte e/2, high nibble = even element; fp32
 * absmax; 16-entry fp32 code) and 1..nsm_lm_head_max_tokens(H) tokens x
 * [tokens][H].  Replaces the GPU NF4 LM head of runtime/lm_head.py:267-468
 * (_materialize_lm_head_nf4_on_gpu + _lm_head_forward's
 * triton_sparse_input_linear_4bit call, :450-468) with the math of its dense
 * head (F.linear on the dequantised weight, :472-480).  H a multiple of 256,
 * quant_block_size a multiple of 64; packed 16-byte, absmax 16-byte (4-byte
 * when quant_block_size > 64) and the workspace 256-byte aligned.  x, bias and out may be fp32 / fp16 / bf16;
 * accumulation is fp32 (fp16 weights x power-of-two-scaled fp16 x on the
 * tensor cores, the absmax applied per 64 columns in fp32). */
size_t nsm_lm_head_workspace_bytes(int32_t tokens, int32_t out_features, int32_t in_features);
int nsm_lm_head_max_tokens(int32_t in_features);
int nsm_lm_head_nf4(const void* x, int32_t x_dtype, int32_t tokens, const uint8_t* packed, const float* absmax,
                    const float* code, int32_t out_features, int32_t in_features, int32_t quant_block_size,
                    const void* bias, int32_t bias_dtype, void* out, int32_t out_dtype, void* workspace,
                    size_t workspace_bytes, nsm_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* NSM_H_ */
