/*
 * hilberta_b200 — C ABI of the B200 (sm_100a) HilbertA inference attention path.
 *
 * Plain pointers, sizes and a CUDA stream (passed as void*); no torch types.
 * Every function returns 0 on success or a negative HB_ERR_* code; none of them
 * allocates or frees device memory (callers pass every buffer) and none of them
 * synchronises the stream except where stated.  Device pointers must be on the
 * current CUDA device.
 *
 * Reference interfaces replaced (wenboluu/hilberta, path:line):
 *   hb_hilbert_order               hilberta/geometry.py:6-25 (hilbert_order)
 *   hb_plan_dims / hb_plan_build   hilberta/plan.py:114-197 (build_plan),
 *                                  hilberta/bridge_k.py:10-51 (bridge_k_plan),
 *                                  hilberta/geometry.py:6-43 (hilbert_order, neighbor_pairs)
 *   hb_validate_metadata           hilberta/sparse_kernel.py:100-152 (validate_metadata)
 *   hb_pair_metadata               hilberta/paired_metadata.py:26-51 (pair_metadata)
 *   hb_dense_mask                  hilberta/plan.py:70-84 (AttentionPlan.dense_mask),
 *                                  hilberta/sparse_kernel.py:155-166 (explicit_mask)
 *   hb_paired_fwd                  hilberta/paired_kernel.py:18-94 (_paired_fwd Triton kernel)
 *                                  launched by paired_kernel.py:97-205 (paired_attention)
 *   hb_norm_rope_pack              hilberta/flux_adapter.py:280-298 (norm_q/norm_k,
 *                                  text+image cat, apply_rotary_emb, BNHD views)
 *   hb_paired_fwd_raster           the same kernel on raster-order tensors, replacing the
 *                                  reorder passes of hilberta/sampling_layout.py:88-116
 *   hb_paired_fwd_allgather        the same kernel fused with the head-output gather
 *                                  before to_out (hilberta/flux_adapter.py:328-339)
 *   hb_expand_kv128                KV128 paired metadata (hilberta/paired_metadata.py:26-51,
 *                                  key_block_size=128) as the equivalent KV64 table
 *   hb_adaln_residual              the adaLN-Zero modulation / gated residual of the FLUX
 *                                  blocks around the processor of flux_adapter.py:259-340
 */
#ifndef HILBERTA_B200_H
#define HILBERTA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define HB_OK 0
#define HB_ERR_ARG -1          /* invalid argument (ValueError in the Python layer)      */
#define HB_ERR_ALIGN -2        /* block/tile alignment precondition violated             */
#define HB_ERR_SHARED -3       /* shared square is not a union of complete blocks        */
#define HB_ERR_CROSS -4        /* a physical block crosses a tile boundary               */
#define HB_ERR_CUDA -5         /* a CUDA runtime call failed                             */
#define HB_ERR_WORKSPACE -6    /* workspace too small                                    */
#define HB_ERR_UNSUPPORTED -7  /* shape/dtype outside the compiled kernels               */
#define HB_ERR_DEVICE -8       /* kernel-reported device status (see hb_fwd_status_*)    */
#define HB_ERR_TMA -9          /* tensor-map encoding rejected the strides/alignment     */

/* device status bits written by hb_paired_fwd into workspace[2] */
#define HB_DEV_TIMEOUT 1       /* a bounded barrier wait ran out; the kernel returned    */
#define HB_DEV_BAD_COUNT 2     /* kv_counts entry outside [0, W]; clamped                */
#define HB_DEV_BAD_BLOCK 4     /* kv_indices entry outside [0, N/64); its tile read zeros */
#define HB_DEV_PEER_TIMEOUT 8  /* hb_paired_fwd_allgather: a peer's completion flag never came */
#define HB_DEV_SMEM_ALIGN 16   /* shared memory not 1024-byte aligned: nothing computed      */

/* Human-readable text for a status code (static storage). */
const char* hb_status_string(int code);

/* Library/ABI version: major*10000 + minor*100 + patch. */
int hb_version(void);

/* ---- metadata builder -------------------------------------------------- */
/* Raster id of the d-th cell of the Hilbert walk, vertically flipped, for
 * d in [0, grid^2) (geometry.py:6-25).  out: int64 [grid^2] on the device. */
int hb_hilbert_order(int grid_size, int64_t* out, void* stream);

typedef struct hb_plan_dims_t {
    int64_t image_tokens;    /* n = grid^2                                          */
    int64_t image_blocks;    /* nb = n / block                                      */
    int64_t total_blocks;    /* (text + n) / block                                  */
    int64_t text_blocks;     /* text / block                                        */
    int64_t shared_blocks;   /* blocks of the shared square (0 when shared == 0)    */
    int64_t rows;            /* ordinary query blocks = nb - shared_blocks          */
    int64_t row_capacity;    /* kv_indices row stride the builder writes (= total)  */
    int64_t workspace_bytes; /* scratch hb_plan_build needs                         */
} hb_plan_dims_t;

/* Host-only: validate the build_plan preconditions (plan.py:117-132) and size
 * the outputs.  HB_ERR_ARG for non-positive / non-power-of-two / grid < 8,
 * HB_ERR_ALIGN for the tile-quarter / text alignment rule. */
int hb_plan_dims(int grid_size, int tile_count, int text_tokens, int block_size, int shared,
                 hb_plan_dims_t* out);

/* Build a plan on the device.
 *   bridge_k  : 0 = no bridge (build_plan bridge=False), 1..4 = top-K bridges.
 *   reciprocal: 0 = build_plan semantics (K must be 0 or 1, directed bridge),
 *               1 = bridge_k_plan semantics (adjacency closed under transpose).
 * Outputs (device, caller-allocated):
 *   image_order, inverse_image_order, original_order : int64 [n]
 *   physical_original_blocks                          : int64 [nb]
 *   kv_indices : int32 [4][rows][row_capacity] (ascending ids, zero padded)
 *   kv_counts  : int32 [4][rows]
 *   bridge_original_blocks : int64 [4][nb][max(1,bridge_k)] (-1 padded)
 *   info       : int32 [8]  ([0] status (HB_ERR_SHARED/HB_ERR_CROSS or 0),
 *                            [1] shared block count, [2..5] max kv count per phase)
 * Enqueued on `stream`; the caller synchronises before reading info. */
int hb_plan_build(int grid_size, int tile_count, int text_tokens, int block_size, int shared,
                  int bridge_k, int reciprocal, int64_t* image_order, int64_t* inverse_image_order,
                  int64_t* original_order, int64_t* physical_original_blocks, int32_t* kv_indices,
                  int32_t* kv_counts, int64_t* bridge_original_blocks, int32_t* info,
                  void* workspace, size_t workspace_bytes, void* stream);

/* Device-side validate_metadata (sparse_kernel.py:100-152) for 64-token blocks.
 * kv_indices int32 [rows][ld], kv_counts int32 [rows].  result[0] receives
 * INT32_MAX when valid, else row*4 + code with code 1 = count outside [1, width],
 * 2 = out-of-range or duplicate id, 3 = a global-prefix block missing (the first
 * failing row, first failing check, in the reference's order).  result[1..3]
 * receive min count, max count and the sum of counts.  `result` must be
 * initialised by hb_validate_metadata itself (it writes the identities first). */
int hb_validate_metadata(const int32_t* kv_indices, int64_t ld, int32_t width, const int32_t* kv_counts,
                         int32_t rows, int32_t tokens, int32_t global_tokens, int32_t* result,
                         void* stream);

/* Paired metadata (paired_metadata.py:26-51) of already-validated rows.
 * out_ids / out_flags int32 [rows/2][ld_out] (zero padded), out_counts int32 [rows/2],
 * info[0] <- max paired count.  key_block_size 64 or 128. */
int hb_pair_metadata(const int32_t* kv_indices, int64_t ld, const int32_t* kv_counts, int32_t rows,
                     int32_t tokens, int32_t global_tokens, int32_t key_block_size, int32_t* out_ids,
                     int32_t* out_flags, int64_t ld_out, int32_t* out_counts, int32_t* info,
                     void* stream);

/* Token-level bool mask [tokens][tokens] (uint8 0/1) of 64-token (block_size) rows:
 * rows < global_tokens all 1, ordinary rows their listed blocks (plan.py:70-84). */
int hb_dense_mask(const int32_t* kv_indices, int64_t ld, const int32_t* kv_counts, int32_t rows,
                  int32_t tokens, int32_t global_tokens, int32_t block_size, uint8_t* mask,
                  void* stream);

/* ---- paired block-sparse attention forward ------------------------------ */
/* Bytes of the per-stream scheduler workspace hb_paired_fwd needs.  It must be
 * zeroed once before first use; the kernel leaves it zeroed (self-resetting)
 * except for the status word workspace[2], which accumulates HB_DEV_* bits until
 * the caller clears it.  Launches that may overlap on the device must use
 * different workspaces. */
size_t hb_fwd_workspace_bytes(void);

/* Workspace bytes with which hb_paired_fwd splits the global pair-rows (every
 * key block) into chunks of ~32 key blocks that run on different SMs and are
 * merged by the last chunk (fp32 O/m/l partials + one counter per global
 * pair-row); 0 for an invalid shape.  Any larger workspace splits too; a
 * smaller one (at least hb_fwd_workspace_bytes()) runs those rows unsplit.
 * Zero it once, like the minimal workspace; the kernel leaves the counters at
 * zero.  The counters sit in a region sized by workspace_bytes alone, so one
 * workspace serves launches of any shape as long as every launch passes the
 * same workspace_bytes for it.  After HB_DEV_TIMEOUT, zero it again. */
size_t hb_fwd_workspace_bytes_for(int B, int H, int N, int G, int D);

/* O = softmax(Q K^T * scale | mask) V over the paired metadata, one launch.
 *   q,k,v,out : [B][H][N][D] with element strides strides[t*3 + {0,1,2}] = (b,h,n)
 *               for t = 0 q, 1 k, 2 v, 3 out; the D stride is 1.
 *   dtype     : 0 = fp16, 1 = bf16.   D: 64 or 128.   key_block_size: 64.
 *   G         : global (fully connected) query prefix, a multiple of 128, < N.
 *   kv_indices/kv_flags int32 [(N-G)/128][W], kv_counts int32 [(N-G)/128]
 *               (device, contiguous, validated).
 *   scale_log2 = softmax scale * log2(e).
 * Global rows (< G) attend every key block; ordinary pair-rows their listed
 * blocks, each flag bit h unmasking query half h.  Asynchronous on `stream`. */
int hb_paired_fwd(const void* q, const void* k, const void* v, void* out, const int64_t* strides,
                  int B, int H, int N, int D, int G, int W, int key_block_size,
                  const int32_t* kv_indices, const int32_t* kv_flags, const int32_t* kv_counts,
                  float scale_log2, int dtype, const int32_t* row_map, void* workspace,
                  size_t workspace_bytes, void* stream);
/* row_map (optional, NULL = identity; device int32 [N], 16-byte aligned): fused
 * token permutation.  Physical token p — the order the metadata indexes (text
 * prefix, then image tokens in Hilbert / packed order) — is read from row
 * row_map[p] of Q, K and V and written to row row_map[p] of out, so callers can
 * keep Q/K/V/O in raster token order (row_map = [0..T) ++ T + image_order,
 * hilberta/plan.py:147) and no separate reorder pass
 * (hilberta/sampling_layout.py:88-116) touches HBM.  Rows are gathered with TMA
 * tile::gather4 (4 rows per instruction); Q/K/V outer strides must then be
 * multiples of D. */

/* ---- raster-order tensors, block by block ------------------------------- */
/* Same computation as hb_paired_fwd for Q/K/V/O kept in raster token order:
 * the first text_tokens tokens in physical order, then a grid x grid image in
 * row-major order (N = text_tokens + grid^2).  The plan's physical image order
 * (hilberta/plan.py:133-150, :192) walks each 64-token block over one aligned
 * 8x8 square of the image, so block b is loaded as one 8x8 box per tile and
 * its output rows are written back into the same square — the reference's
 * reorder passes before and after the transformer (sampling_layout.py:88-116)
 * are not needed.  block_origin: device int32 [grid^2 / 64], the image row
 * (y0 * grid + x0) of the square physical image block b covers.  A block
 * whose origin is not the corner of an aligned square reads zeros, its rows
 * are not written, and HB_DEV_BAD_BLOCK is set.  Within a block, keys and
 * queries are taken in the square's row-major order, so results equal
 * hb_paired_fwd's on tensors permuted to that order (the same values up to
 * the order of fp32 sums otherwise). */
typedef struct hb_raster_order_t {
    int32_t text_tokens;          /* multiple of 64                              */
    int32_t grid;                 /* image side, multiple of 8                   */
    const int32_t* block_origin;  /* device, [grid * grid / 64]                  */
} hb_raster_order_t;
int hb_paired_fwd_raster(const void* q, const void* k, const void* v, void* out,
                         const int64_t* strides, int B, int H, int N, int D, int G, int W,
                         int key_block_size, const int32_t* kv_indices, const int32_t* kv_flags,
                         const int32_t* kv_counts, float scale_log2, int dtype,
                         const hb_raster_order_t* order, void* workspace, size_t workspace_bytes,
                         void* stream);

/* ---- attention fused with the all-gather of head outputs --------------- */
/* Head-parallel ranks (one process per GPU, the heads split over the ranks;
 * the gather the FLUX block does before to_out, hilberta/flux_adapter.py:328-339)
 * need every rank's output heads on every rank.  Instead of the kernel followed
 * by an all-gather, hb_paired_fwd_allgather writes each finished output row
 * straight into every rank's full-head output over NVLink peer memory (plain
 * stores into mappings from hb_ipc_open), so the transfer overlaps the math tile
 * by tile.  When all of this rank's rows are stored it fences at system scope,
 * sets its word in every rank's flag array to `epoch` and waits (bounded by
 * timeout_ms; on expiry HB_DEV_PEER_TIMEOUT) until every rank has set its word
 * in this rank's array: when the launch completes, all ranks' rows are in this
 * rank's output.  The ranks must be on distinct GPUs.  A rank must not write a
 * buffer a peer may still read: alternate two output buffers between calls (a
 * rank reaches call e+1 only after every rank finished call e's kernel, hence
 * everything it ordered before that kernel). */
#define HB_MAX_RANKS 8
typedef struct hb_peer_out_t {
    int32_t n_ranks;               /* 1..HB_MAX_RANKS                                   */
    int32_t rank;                  /* this rank: its word in every flag array            */
    int32_t epoch;                 /* > 0, the same on all ranks, +1 per call            */
    int32_t timeout_ms;            /* bound of the completion wait; 0 = 10000            */
    void* out[HB_MAX_RANKS];       /* rank i's output at this rank's first head, strides
                                      strides[9..11] (identical on all ranks)           */
    int32_t* flags[HB_MAX_RANKS];  /* rank i's HB_MAX_RANKS flag words, zeroed once     */
} hb_peer_out_t;
/* Same arguments as hb_paired_fwd with `out` and `row_map` replaced by `peers`. */
int hb_paired_fwd_allgather(const void* q, const void* k, const void* v, const int64_t* strides,
                            int B, int H, int N, int D, int G, int W, int key_block_size,
                            const int32_t* kv_indices, const int32_t* kv_flags,
                            const int32_t* kv_counts, float scale_log2, int dtype,
                            const hb_peer_out_t* peers, void* workspace, size_t workspace_bytes,
                            void* stream);

/* Peer mappings for hb_peer_out_t (CUDA IPC; no multicast objects).
 * hb_ipc_export: handle (HB_IPC_HANDLE_BYTES) of the device allocation holding
 * ptr, and ptr's byte offset in it.  hb_ipc_open (another process, same node):
 * maps that allocation on the current device and returns base + offset;
 * hb_ipc_close unmaps what hb_ipc_open returned (pass the same offset). */
#define HB_IPC_HANDLE_BYTES 64
int hb_ipc_export(const void* ptr, void* handle, uint64_t* offset);
int hb_ipc_open(const void* handle, uint64_t offset, void** ptr);
int hb_ipc_close(void* ptr, uint64_t offset);
/* One plain device-to-device copy of `bytes` (cudaMemcpyAsync on `stream`);
 * `dst` may be a mapping from hb_ipc_open.  No counterpart in the reference
 * (it has no multi-GPU path): the copy-engine transfer into a peer's memory
 * that callers time to know the NVLink bandwidth the fused all-gather's peer
 * stores are held against. */
int hb_peer_copy(void* dst, const void* src, size_t bytes, void* stream);
/* `bytes` from `src` to each of the n_dst destinations (1..HB_MAX_RANKS; any of
 * them may be hb_ipc_open mappings) by SM stores: two CTAs per SM, each lane
 * loading 16 bytes and storing them to every destination, consecutive lanes on
 * consecutive 16-byte chunks (the store pattern of the fused all-gather's peer
 * copies).  Pointers 16-byte aligned, bytes a multiple of 16.  No counterpart
 * in the reference: callers time it to know the NVLink bandwidth those stores
 * reach when every rank sends at once. */
int hb_peer_scatter(const void* src, void* const* dst, int n_dst, size_t bytes, void* stream);

/* ---- Q/K/V preparation before the attention ----------------------------- */
/* The FLUX processor's steps between the projections and the attention
 * (hilberta/flux_adapter.py:280-298), for one of Q, K or V, in one pass over
 * HBM: split into H heads of D, RMS-normalise each (token, head) row over D with
 * a learned weight (w_txt for the text stream, w_img for the image stream; both
 * NULL: no normalisation, as for V), put the T text tokens first, rotate pairs
 * (2i, 2i+1) by the rotary embedding (cos/sin NULL: no rotation) and write
 * out[b][s][h][:] (element strides o_sb, o_sn, o_sh; [B, S, H, D] storage is
 * what the attention reads in place through [B, H, S, D] views).
 *   txt [B][T][H*D], img [B][n][H*D]: 16-bit (dtype 0 fp16, 1 bf16) with element
 *   strides (txt_sb, txt_sn), (img_sb, img_sn); weights [D] in the same dtype;
 *   cos/sin fp32 [T+n][D] indexed by OUTPUT token.  image_rows (optional, device
 *   int32 [n]): image token i is written to token T + image_rows[i] (e.g. the
 *   plan's inverse order, to produce the physical layout); an entry outside
 *   [0, n) drops that row and sets HB_DEV_BAD_BLOCK in *status (optional).
 * The rounding follows the ops it replaces (diffusers 0.36 RMSNorm and
 * apply_rotary_emb): fp32 mean of squares, round to 16 bits after x*rsqrt and
 * after *weight, rotation as separately rounded fp32 products and sum.
 * Pointers 16-byte aligned, strides multiples of 8 elements; D 64 or 128. */
int hb_norm_rope_pack(const void* txt, int64_t txt_sb, int64_t txt_sn, const void* img,
                      int64_t img_sb, int64_t img_sn, int B, int T, int n, int H, int D,
                      const void* w_txt, const void* w_img, float eps, const float* cos,
                      const float* sin, const int32_t* image_rows, void* out, int64_t o_sb,
                      int64_t o_sn, int64_t o_sh, int dtype, int32_t* status, void* stream);

/* ---- KV128 paired metadata -> KV64 -------------------------------------- */
/* The reference kernel also takes paired metadata with 128-key blocks
 * (paired_metadata.py:26-51 key_block_size=128: flag bit half + 2*key_half;
 * paired_kernel.py:65-75).  hb_paired_fwd runs 64-key blocks; this rewrites a
 * KV128 table [rows][ld] (width used entries per row) into the equivalent KV64
 * table [rows][ld_out] (ld_out >= 2*width; entries past a row's count are not
 * written): entry (b, f) becomes (2b, f & 3) and (2b+1, (f >> 2) & 3), each only
 * when its bits are nonzero, in order.  The result equals pair_metadata with
 * key_block_size 64 on the same rows, so the attention is the same. */
int hb_expand_kv128(const int32_t* kv_indices, const int32_t* kv_flags, int64_t ld, int32_t width,
                    const int32_t* kv_counts, int32_t rows, int32_t* out_ids, int32_t* out_flags,
                    int64_t ld_out, int32_t* out_counts, void* stream);

/* ---- adaLN modulation and gated residual of the FLUX blocks -------------- */
/* No counterpart in the reference's own code: the adaLN-Zero steps of the
 * diffusers FLUX blocks that call the attention processor
 * (hilberta/flux_adapter.py:259-340 wraps that processor), fused:
 *   x' = x + gate[b] * y                              (when y is given)
 *   h  = LayerNorm(x') * (1 + scale[b]) + shift[b]    (when h_out is given)
 * over `rows` rows of C elements, row r in batch b = r / rows_per_batch.
 * x, y, x_out, h_out: 16-bit (dtype 0 fp16, 1 bf16) rows with element row
 * strides x_rs, y_rs, xo_rs, h_rs (x_out may alias x); gate/shift/scale: [B][C]
 * with batch stride mod_bs, unit element stride.  LayerNorm without affine
 * weights, eps as given; fp32 arithmetic, x' rounded to 16 bits before the
 * LayerNorm, h rounded once.  C a multiple of 256 up to 4096; pointers 16-byte
 * aligned, strides multiples of 8 elements. */
int hb_adaln_residual(const void* x, int64_t x_rs, const void* y, int64_t y_rs, const void* gate,
                      const void* shift, const void* scale, int64_t mod_bs, void* x_out,
                      int64_t xo_rs, void* h_out, int64_t h_rs, int rows, int rows_per_batch, int C,
                      float eps, int dtype, void* stream);

/* ---- allocation-free variant of hb_paired_fwd --------------------------- */
/* No counterpart in the reference: an addition for callers that must not
 * allocate device memory.  Some hosts cannot call cudaMalloc from the thread
 * that enqueues work: plugin interfaces of inference runtimes that own every
 * device allocation and forbid allocating while enqueueing, real-time services
 * that fix their memory budget at start-up, and language bindings that have no
 * CUDA allocator to hand the per-stream workspace hb_paired_fwd expects.
 *
 * Same arguments and result as hb_paired_fwd, minus `workspace`: the scheduler
 * words live in a library-owned static device array of
 * HB_NOALLOC_SCRATCH_BYTES bytes, one per GPU that loads the library, held
 * until the process exits.  The first call on a device looks the array's
 * address up (cudaGetSymbolAddress, with that device current); make that first
 * call before any stream capture.  Each call clears the words it uses
 * (cudaMemsetAsync, no allocation) and then launches the same kernel as
 * hb_paired_fwd.  All calls share the one array, so calls that may overlap on
 * the GPU (different streams, no ordering between them) race; serialise them
 * or use hb_paired_fwd with separate workspaces.  Device status bits are not
 * reported by this variant.  Problems needing more than HB_NOALLOC_MAX_ITEMS
 * (2^30 - 1) work items (B*H*N/128) are rejected with HB_ERR_UNSUPPORTED before
 * any CUDA call; that is the same bound the kernel's scheduler has. */
#define HB_NOALLOC_SCRATCH_BYTES 256
#define HB_NOALLOC_MAX_ITEMS ((1 << 30) - 1)
int hb_paired_fwd_noalloc(const void* q, const void* k, const void* v, void* out,
                          const int64_t* strides, int B, int H, int N, int D, int G, int W,
                          int key_block_size, const int32_t* kv_indices, const int32_t* kv_flags,
                          const int32_t* kv_counts, float scale_log2, int dtype, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* HILBERTA_B200_H */
