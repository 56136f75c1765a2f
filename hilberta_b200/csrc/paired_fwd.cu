// Paired block-sparse flash-attention forward for B200 (sm_100a).
//
// Computes, for every (batch, head) and every 128-query pair-row, the online-
// softmax attention over the pair-row's listed 64-key blocks, each block's flag
// bit h unmasking query half h (rows 64h..64h+63) — the computation of the
// reference Triton kernel hilberta/paired_kernel.py:18-94 (global pair-rows,
// rows < G, visit every key block with both flags set, paired_kernel.py:52-57,
// 71-75; ALL_QUERIES mode).
//
// B200 design (one CTA = 8 warps, two CTAs per SM, persistent):
//   warp 0  item fetcher (atomic work counter; global-row chunks first, then
//           ordinary pair-rows head-major): decodes each item and its first 32
//           flags into a two-slot shared ring; TMA loads of Q and K (3 stages)
//   warp 1  TMA loads of V (2 stages)
//   warp 2  single-thread tcgen05.mma issuer: S = Q K^T (SS, 128x64x16 steps)
//           into TMEM, O += P V (TS: P read from TMEM, V MN-major from SMEM),
//           each issued as soon as its inputs are ready (non-blocking polls)
//   warp 3  TMEM allocator; in the fused all-gather, pushes rows to the peers
//   warps 4-7  softmax: one TMEM lane (query row) per thread, exp2 online
//           softmax with lazy O rescaling (only when the running max grows by
//           more than 2^8), P written back into the S columns as 16-bit pairs.
//           An item's epilogue (O / l -> the output with 32-byte stores, or the
//           fused all-gather's hand-off, or a chunk's partial for split rows)
//           runs after the NEXT item's first step, when its last PV has long
//           completed and the next first PV is the only MMA waiting for O.
// TMEM per CTA: S0 [0,64) S1 [64,128) O [128,128+D) (256 columns; two CTAs fill
// the 512-column TMEM of an SM).  Tiles use the 128-byte swizzle end to end;
// mbarriers live after the tiles in the (1024-byte aligned) dynamic region.
// Token layouts (template MODE): physical order (tiled maps), any permutation
// (row map, tile::gather4), raster order by 8x8 image squares (5-D maps).
// Every mbarrier wait is bounded; a timeout sets HB_DEV_TIMEOUT and the CTA
// drains and exits instead of hanging.  No cluster multicast anywhere.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "sm100_ptx.cuh"

namespace hb {
namespace {

using namespace ptx;
constexpr unsigned FULL = 0xffffffffu;

struct FwdParams {
    CUtensorMap tmap_q;
    CUtensorMap tmap_k;
    CUtensorMap tmap_v;
    int32_t perm_q[3], perm_k[3], perm_v[3];  // tensor-map dim (1..3) holding (n, h, b)
    int64_t o_sb, o_sh, o_sn;
    const int32_t* indices;
    const int32_t* flags;
    const int32_t* counts;
    int32_t* ws;  // [0] next work item, [1] finished CTAs, [2] status bits
    int B, H, N, G, W;
    int g_rows;          // G / 128 global pair-rows
    int o_rows;          // (N - G) / 128 ordinary pair-rows
    int n_global_items;    // items of the global chunks scheduled first: B * H * g_rows * head_chunks
    int n_ordinary_items;  // B * H * o_rows, scheduled next
    int num_items;         // then B * H * g_rows * tail_chunks tail chunks
    int nkb;  // N / 64 key blocks
    // Split of the global pair-rows over their key blocks (n_chunks == 1: none).
    // Head chunk c < head_chunks covers blocks [c*chunk, min(head_blocks,
    // (c+1)*chunk)); tail chunk t < tail_chunks covers tail_blocks blocks from
    // head_blocks + t*tail_blocks and runs after every ordinary pair-row (short
    // items at the end of the launch even out the CTAs' finishing times).  Each
    // chunk leaves O, m, l of its 128 rows in `partial`; the last to finish merges.
    int chunk, n_chunks;  // head chunk size; head_chunks + tail_chunks
    int head_chunks, head_blocks, tail_chunks, tail_blocks;
    float* partial;      // [B*H*g_rows][n_chunks][128*D + 256] fp32
    int32_t* chunk_cnt;  // [B*H*g_rows] finished chunks (reset to 0 by the merger)
    // Fused token permutation: physical token p of the layout the metadata indexes
    // reads and writes source row row_map[p] of Q/K/V/O (null: identity).  The
    // gathered tensor maps are 2-D (D, rows); rs_* = (b, h, n) strides in rows.
    const int32_t* row_map;
    int64_t rs_q[3], rs_k[3], rs_v[3];
    // MODE_SQUARES: tokens < 64*text_blocks are in physical order (text maps above,
    // 64-row boxes); image block ib covers the 8x8 square whose top-left token is
    // image row sq_origin[ib] (= y0*grid + x0), loaded through the 5-D maps
    // (D, x, y, head, batch) based at the first image token.
    CUtensorMap tmap_q_img, tmap_k_img, tmap_v_img;
    int text_blocks, grid, img_blocks;
    const int32_t* sq_origin;
    // Output rows go to n_out tensors (same strides o_s*): `out` alone, or every
    // rank's full-head output at this rank's first head (fused all-gather).  In
    // the latter mode (n_out > 1) the last CTA signals flags[i][rank] = epoch on
    // every rank i and waits for flags[rank][i] from all of them.
    int n_out, rank, epoch;
    void* outs[HB_MAX_RANKS];
    int32_t* peer_flags[HB_MAX_RANKS];
    long long peer_timeout;  // SM cycles the completion wait may take
    float scale_log2;
    long long timeout;  // SM cycles a single barrier wait may take
};

// Scratch layout of the workspace, in bytes: header (scheduler words), chunk
// counters, then the chunk partials.  The counter region's size depends only on
// the workspace size (room for every group a split launch could fit), so the
// partials of one launch never overlap the counters of a launch with more groups
// that uses the same workspace: the counters stay zero between launches.
constexpr int64_t WS_HEADER = 256;
constexpr int MAX_CHUNKS = 32;
constexpr int CHUNK_BLOCKS = 32;                          // target key blocks per chunk of a global pair-row
constexpr int TAIL_CHUNKS = 2;  // short chunks of an unsplit global row, run at the end of the launch
constexpr int64_t MIN_GROUP_PARTIAL = 2 * (128 * 64 + 256) * 4;  // smallest partials of one split group
inline int64_t counter_bytes(int64_t ws) { return ((4 * (ws / MIN_GROUP_PARTIAL + 1) + 255) / 256) * 256; }

// One work item handed from the fetcher (warp 0) to the other roles: its index,
// its block count and, for an ordinary pair-row, the flags of its first 32
// entries, so no consumer makes a dependent global load when an item starts.
struct ItemSlot {
    int item, n;
    int flags[32];
};

template <int D>
struct Cfg {
    static constexpr int SLABS = D / 64;           // 64-element (128-byte) column slabs
    static constexpr int Q_SLAB = 128 * 128;       // 128 rows x 128 B
    static constexpr int KV_SLAB = 64 * 128;       // 64 rows x 128 B
    static constexpr int Q_BYTES = Q_SLAB * SLABS;
    static constexpr int KV_BYTES = KV_SLAB * SLABS;
    static constexpr int KS = 3;  // K stages: a K tile is issued while the two before it are consumed
    static constexpr int VS = 2;  // V stages
    // Mbarriers and slots live after the tiles in the dynamic region (no static
    // shared memory, so the region starts 1024-byte aligned with no padding:
    // two CTAs with three K stages fit in an SM's 228 KB).
    struct Ctl {
        uint64_t q_full, q_empty, o_done, o_empty, drain, wg, final_done;
        uint64_t k_full[KS], k_empty[KS], v_full[VS], v_empty[VS];
        uint64_t s_full[2], p_full[2], item_full[2], item_empty[2];
        uint64_t push_full[2], push_empty[2];  // fused all-gather: finished items handed to warp 3
        ItemSlot slots[2];
        int push_item[2];
        uint32_t tmem_base;
        int abort;
        int wg_flag;
    };
    static constexpr int CTL_OFF = Q_BYTES + (KS + VS) * KV_BYTES;
    static constexpr int SMEM = CTL_OFF + (int)((sizeof(Ctl) + 15) / 16 * 16);
    static constexpr int TMEM_COLS = 256;
    static constexpr uint32_t S_COL0 = 0, O_COL = 128;
};

// Token layouts of Q/K/V/O (kernel template MODE):
//   MODE_TILED    physical order, the layout the metadata indexes (4-D tiled maps)
//   MODE_ROWS     any permutation: row row_map[p] holds physical token p (gather4)
//   MODE_SQUARES  raster order of a text prefix + g x g image whose physical
//                 64-token blocks are aligned 8x8 squares: one 5-D box per block
constexpr int MODE_TILED = 0, MODE_ROWS = 1, MODE_SQUARES = 2;

constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units: P <= 2^8 between rescales

struct Item {
    int b, h, qrow0, row, n;
    int blk0;         // global rows: first key block of this chunk
    int chunk, group; // global rows: chunk index, (b*H + h)*g_rows + global pair-row
    bool global, split;
};

// Work item -> (batch, head, query rows, key blocks), given its block count n
// (pure arithmetic: no loads).
__device__ __forceinline__ Item decode_item_n(const FwdParams& p, int item, int n) {
    Item w;
    const int t_ord = item - p.n_global_items;
    if (item < p.n_global_items || t_ord >= p.n_ordinary_items) {
        // head chunks: (bh, chunk, global pair-row), so the global rows reading
        // the same key blocks of one head run back to back (K/V served from L2);
        // tail chunks likewise, after the ordinary rows
        const bool head = item < p.n_global_items;
        const int t0 = head ? item : t_ord - p.n_ordinary_items;
        const int nc = head ? p.head_chunks : p.tail_chunks;
        const int gp = t0 % p.g_rows;
        const int t = t0 / p.g_rows;
        const int c = t % nc;
        const int bh = t / nc;
        w.b = bh / p.H;
        w.h = bh % p.H;
        w.qrow0 = gp * 128;
        w.row = 0;
        w.blk0 = head ? c * p.chunk : p.head_blocks + c * p.tail_blocks;
        w.chunk = head ? c : p.head_chunks + c;
        w.group = bh * p.g_rows + gp;
        w.global = true;
        w.split = p.n_chunks > 1;
    } else {
        w.blk0 = 0;
        w.chunk = 0;
        w.group = 0;
        w.split = false;
        const int bh = t_ord / p.o_rows;
        w.b = bh / p.H;
        w.h = bh % p.H;
        w.row = t_ord % p.o_rows;
        w.qrow0 = p.G + w.row * 128;
        w.global = false;
    }
    w.n = n;
    return w;
}

// Block count of a work item: a global chunk's from the split, an ordinary
// pair-row's from the metadata (clamped to [1, W]; out of range is reported).
__device__ __forceinline__ int item_blocks(const FwdParams& p, int item, bool report) {
    if (item < p.n_global_items) {
        const int c = (item / p.g_rows) % p.head_chunks;
        return min(p.chunk, p.head_blocks - c * p.chunk);
    }
    const int t_ord = item - p.n_global_items;
    if (t_ord >= p.n_ordinary_items) return p.tail_blocks;
    const int row = t_ord % p.o_rows;
    const int c = p.counts[row];
    if (report && (c < 1 || c > p.W)) atomicOr(&p.ws[2], HB_DEV_BAD_COUNT);
    return c < 1 ? 1 : (c > p.W ? p.W : c);
}

__device__ __forceinline__ void tma_coords(const int32_t* perm, int n, int h, int b, int& c1, int& c2, int& c3) {
    c1 = perm[0] == 1 ? n : (perm[1] == 1 ? h : b);
    c2 = perm[0] == 2 ? n : (perm[1] == 2 ? h : b);
    c3 = perm[0] == 3 ? n : (perm[1] == 3 ? h : b);
}

// All 32 lanes poll in lock step so the warp stays converged for the
// warp-collective tcgen05 loads/stores that follow; bounded like mbar_wait.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, long long limit) {
    long long t0 = 0;
    bool started = false;
    while (true) {
        const bool ok = mbar_try_wait(bar, parity);
        if (__all_sync(FULL, ok)) return true;
        int stop = 0;
        if ((threadIdx.x & 31) == 0) {
            if (!started) {
                t0 = clock64();
                started = true;
            }
            if (*abort_flag || clock64() - t0 > limit) {
                *abort_flag = 1;
                stop = 1;
            }
        }
        if (__shfl_sync(FULL, stop, 0)) return false;
    }
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
    if constexpr (BF16) {
        __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&v);
    } else {
        __half2 v = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&v);
    }
}

// Gather mode: lane i (i < rows/4) loads token rows base+4i..base+4i+3 of a tile
// through the physical -> source row map, one tile::gather4 per 64-column slab
// into 128-byte rows 4i..4i+3 of the tile (the same swizzled layout a tiled load
// gives).  rs = (b, h, n) strides of the tensor in rows of D elements.
template <int D>
__device__ __forceinline__ void gather_tile(const FwdParams& p, const CUtensorMap* map, const int64_t* rs, uint8_t* dst,
                                            int slab_bytes, uint64_t* bar, int base, int rows, int b, int h, bool bad) {
    const int lane = threadIdx.x & 31;
    if (4 * lane >= rows) return;
    const int4 src = *reinterpret_cast<const int4*>(p.row_map + base + 4 * lane);
    const int64_t r0 = (int64_t)b * rs[0] + (int64_t)h * rs[1];
    const int s0 = bad ? -1 : (int)(r0 + (int64_t)src.x * rs[2]);
    const int s1 = bad ? -1 : (int)(r0 + (int64_t)src.y * rs[2]);
    const int s2 = bad ? -1 : (int)(r0 + (int64_t)src.z * rs[2]);
    const int s3 = bad ? -1 : (int)(r0 + (int64_t)src.w * rs[2]);
#pragma unroll
    for (int s = 0; s < D / 64; s++) tma_gather4(dst + s * slab_bytes + 4 * lane * 128, map, bar, 64 * s, s0, s1, s2, s3);
}

// MODE_SQUARES: raster row of image block ib's first token, or -1 when the block
// or its origin is invalid (out of range, or not the corner of an aligned 8x8 square).
__device__ __forceinline__ int square_origin(const FwdParams& p, int ib) {
    if (ib < 0 || ib >= p.img_blocks) return -1;
    const int o = p.sq_origin[ib];
    if (o < 0 || o >= p.grid * p.grid || ((o % p.grid) & 7) || ((o / p.grid) & 7)) return -1;
    return o;
}

// MODE_SQUARES: one 64-token physical block into 64 rows of a swizzled tile (lane
// 0 only): a text block through the 4-D map, an image block as one 8x8 box of
// the 5-D map per 64-column slab.  A bad block reads fully out of bounds (zeros).
template <int D>
__device__ __forceinline__ void load_block_sq(const FwdParams& p, const CUtensorMap* text_map, const int32_t* perm,
                                              const CUtensorMap* img_map, uint8_t* dst, int slab_bytes, uint64_t* bar,
                                              int blk, int b, int h, uint64_t policy) {
    if (blk >= 0 && blk < p.text_blocks) {
        int c1, c2, c3;
        tma_coords(perm, blk * 64, h, b, c1, c2, c3);
#pragma unroll
        for (int s = 0; s < D / 64; s++)
            tma_load_4d_hint(dst + s * slab_bytes, text_map, bar, 64 * s, c1, c2, c3, policy);
        return;
    }
    const int o = square_origin(p, blk - p.text_blocks);
    int x0 = 0, y0 = p.grid;  // y beyond the image: zero fill
    if (o >= 0) {
        x0 = o % p.grid;
        y0 = o / p.grid;
    } else {
        atomicOr(&p.ws[2], HB_DEV_BAD_BLOCK);
    }
#pragma unroll
    for (int s = 0; s < D / 64; s++)
        tma_load_5d_hint(dst + s * slab_bytes, img_map, bar, 64 * s, x0, y0, h, b, policy);
}

// Producer of one operand stream (warp-wide; lane 0 issues, every lane in gather
// mode).  WHICH = 0: Q + K, 1: V.
template <int D, int WHICH, int MODE>
__device__ void producer(const FwdParams& p, uint8_t* sQ, uint8_t* sKV, uint64_t* bar_item_full,
                         uint64_t* bar_item_empty, ItemSlot* slots, uint64_t* bar_q_full, uint64_t* bar_q_empty,
                         uint64_t* bar_full, uint64_t* bar_empty, volatile int* abort_flag) {
    using C = Cfg<D>;
    constexpr int STAGES = WHICH == 0 ? C::KS : C::VS;
    const int lane = threadIdx.x & 31;
    const CUtensorMap* tmap = WHICH == 0 ? &p.tmap_k : &p.tmap_v;
    const int32_t* perm = WHICH == 0 ? p.perm_k : p.perm_v;
    const int64_t* rs = WHICH == 0 ? p.rs_k : p.rs_v;
    uint32_t gx = 0;  // loads issued over this CTA's lifetime
    bool ok = true;
    // L2 priorities: K/V tiles are re-read by every pair-row that lists them,
    // Q tiles are read once (as are the output rows): keep the former, let the
    // latter go first.
    const uint64_t pol_kv = l2_policy_evict_last();
    const uint64_t pol_q = l2_policy_evict_first();
    for (int it = 0; ok; it++) {
        const int slot = it & 1;
        int item;
        Item w;
        if (WHICH == 0) {
            if (!warp_wait(&bar_item_empty[slot], ((it >> 1) & 1) ^ 1, abort_flag, p.timeout)) break;
            item = 0;
            if (lane == 0) item = atomicAdd(&p.ws[0], 1);
            item = __shfl_sync(FULL, item, 0);
            // decode (the block count of an ordinary row) and the first 32 flags
            // before publishing the item: one warp-wide load each
            int n = 0, fl = 0;
            if (item < p.num_items) {
                w = decode_item_n(p, item, item_blocks(p, item, lane == 0));
                n = w.n;
                fl = w.global ? 3 : (lane < w.n ? p.flags[(int64_t)w.row * p.W + lane] : 0);
            }
            slots[slot].flags[lane] = fl;
            if (lane == 0) {
                slots[slot].item = item;
                slots[slot].n = n;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar_item_full[slot]);
        } else {
            if (!warp_wait(&bar_item_full[slot], (it >> 1) & 1, abort_flag, p.timeout)) break;
            item = slots[slot].item;
            const int n = slots[slot].n;
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar_item_empty[slot]);
            if (item < p.num_items) w = decode_item_n(p, item, n);
        }
        if (item >= p.num_items) break;
        if (WHICH == 0) {
            if (!warp_wait(bar_q_empty, (it & 1) ^ 1, abort_flag, p.timeout)) break;
            if constexpr (MODE == MODE_ROWS) {
                if (lane == 0) mbar_arrive_expect_tx(bar_q_full, C::Q_BYTES);
                __syncwarp();
                gather_tile<D>(p, &p.tmap_q, p.rs_q, sQ, C::Q_SLAB, bar_q_full, w.qrow0, 128, w.b, w.h, false);
            } else if constexpr (MODE == MODE_SQUARES) {
                if (lane == 0) {
                    mbar_arrive_expect_tx(bar_q_full, C::Q_BYTES);
                    for (int half = 0; half < 2; half++)  // query half = one physical block
                        load_block_sq<D>(p, &p.tmap_q, p.perm_q, &p.tmap_q_img, sQ + half * 64 * 128, C::Q_SLAB,
                                         bar_q_full, (w.qrow0 >> 6) + half, w.b, w.h, pol_q);
                }
            } else if (lane == 0) {
                mbar_arrive_expect_tx(bar_q_full, C::Q_BYTES);
                int c1, c2, c3;
                tma_coords(p.perm_q, w.qrow0, w.h, w.b, c1, c2, c3);
#pragma unroll
                for (int s = 0; s < C::SLABS; s++)
                    tma_load_4d_hint(sQ + s * C::Q_SLAB, &p.tmap_q, bar_q_full, 64 * s, c1, c2, c3, pol_q);
            }
        }
        int chunk = 0;
        for (int j = 0; j < w.n; j++, gx++) {
            if (!w.global && (j & 31) == 0) {
                const int jj = j + lane;
                chunk = jj < w.n ? p.indices[(int64_t)w.row * p.W + jj] : 0;
            }
            const int blk = w.global ? w.blk0 + j : __shfl_sync(FULL, chunk, j & 31);
            const int st = gx % STAGES;
            if (!warp_wait(&bar_empty[st], ((gx / STAGES) & 1) ^ 1, abort_flag, p.timeout)) {
                ok = false;
                break;
            }
            const bool bad = blk < 0 || blk >= p.nkb;
            if constexpr (MODE == MODE_ROWS) {
                if (lane == 0) {
                    if (bad) atomicOr(&p.ws[2], HB_DEV_BAD_BLOCK);
                    mbar_arrive_expect_tx(&bar_full[st], C::KV_BYTES);
                }
                __syncwarp();
                // a bad block reads row -1: out of bounds, the TMA unit fills zeros
                gather_tile<D>(p, tmap, rs, sKV + st * C::KV_BYTES, C::KV_SLAB, &bar_full[st], bad ? 0 : blk * 64, 64,
                               w.b, w.h, bad);
            } else if constexpr (MODE == MODE_SQUARES) {
                if (lane == 0) {
                    if (bad) atomicOr(&p.ws[2], HB_DEV_BAD_BLOCK);
                    mbar_arrive_expect_tx(&bar_full[st], C::KV_BYTES);
                    load_block_sq<D>(p, tmap, perm, WHICH == 0 ? &p.tmap_k_img : &p.tmap_v_img,
                                     sKV + st * C::KV_BYTES, C::KV_SLAB, &bar_full[st], bad ? -1 : blk, w.b, w.h,
                                     pol_kv);
                }
            } else if (lane == 0) {
                int rowc = blk * 64;
                if (bad) {
                    rowc = p.N;  // fully out of bounds: the TMA unit fills zeros
                    atomicOr(&p.ws[2], HB_DEV_BAD_BLOCK);
                }
                mbar_arrive_expect_tx(&bar_full[st], C::KV_BYTES);
                int c1, c2, c3;
                tma_coords(perm, rowc, w.h, w.b, c1, c2, c3);
#pragma unroll
                for (int s = 0; s < C::SLABS; s++)
                    tma_load_4d_hint(sKV + st * C::KV_BYTES + s * C::KV_SLAB, tmap, &bar_full[st], 64 * s, c1, c2, c3,
                                     pol_kv);
            }
        }
    }
    if (*abort_flag) {
        // Let TMA copies already in flight land in this CTA's shared memory.
        const long long t0 = clock64();
        while (clock64() - t0 < (1ll << 22)) {
        }
    }
}

template <int D, bool BF16>
__device__ void mma_issuer(const FwdParams& p, uint32_t tmem, uint8_t* sQ, uint8_t* sK, uint8_t* sV,
                           uint64_t* bar_item_full, uint64_t* bar_item_empty, ItemSlot* slots, uint64_t* bar_q_full,
                           uint64_t* bar_q_empty, uint64_t* bar_k_full, uint64_t* bar_k_empty, uint64_t* bar_v_full,
                           uint64_t* bar_v_empty, uint64_t* bar_s_full, uint64_t* bar_p_full, uint64_t* bar_o_done,
                           uint64_t* bar_o_empty, uint64_t* bar_drain, uint64_t* bar_final, volatile int* abort_flag) {
    using C = Cfg<D>;
    constexpr uint32_t IDESC_QK = idesc_f16(128, 64, BF16, false);
    constexpr uint32_t IDESC_PV = idesc_f16(128, D, BF16, true);
    // Descriptor bases built once; each MMA adds a compile-time (offset >> 4) to
    // the 14-bit start-address field (shared addresses stay below 2^18, so the
    // field never carries).
    const uint64_t dq0 = desc_sw128(smem_u32(sQ), 16, 1024);
    const uint64_t dk0 = desc_sw128(smem_u32(sK), 16, 1024);
    const uint64_t dv0 = desc_sw128(smem_u32(sV), C::KV_SLAB, 1024);
    uint32_t g = 0, gk = 0, gv = 0;
    bool ok = true;
    for (int it = 0; ok; it++) {
        const int slot = it & 1;
        if (!mbar_wait(&bar_item_full[slot], (it >> 1) & 1, abort_flag, p.timeout)) break;
        const int item = slots[slot].item;
        const int n_item = slots[slot].n;
        mbar_arrive(&bar_item_empty[slot]);
        if (item >= p.num_items) {
            tc_commit(bar_final);  // completes once every MMA issued by this CTA has
            break;
        }
        const Item w = decode_item_n(p, item, n_item);
        if (!mbar_wait(bar_q_full, it & 1, abort_flag, p.timeout)) break;
        tc_fence_after();
        // Issue S_js = Q K_js^T and O += P_jp V_jp in whichever order their inputs
        // arrive (S first when both can go): a late K tile then no longer holds
        // back a PV whose P and V are ready.  S_js reuses the TMEM buffer of
        // P_{js-2}, so it waits until PV_{js-2} is issued (the MMAs run in issue
        // order).  A phase seen complete cannot advance before it is consumed
        // (its next arrival needs this issue first), so polling is exact.
        int js = 0, jp = 0;
        bool o_free = false;  // the previous item's epilogue has read O
        long long t0 = 0;
        bool waiting = false;
        while (jp < w.n) {
            bool issued = false;
            if (js < w.n && jp >= js - 1) {
                const int st = gk % C::KS;
                if (mbar_test_wait(&bar_k_full[st], (gk / C::KS) & 1)) {
                    tc_fence_after();
                    const uint32_t d_s = tmem + C::S_COL0 + ((g + js) & 1) * 64;
                    const uint64_t dk_st = dk0 + (uint64_t)((st * C::KV_BYTES) >> 4);
#pragma unroll
                    for (int kk = 0; kk < D / 16; kk++) {
                        const uint64_t a = dq0 + (uint64_t)(((kk >> 2) * C::Q_SLAB + (kk & 3) * 32) >> 4);
                        const uint64_t b = dk_st + (uint64_t)(((kk >> 2) * C::KV_SLAB + (kk & 3) * 32) >> 4);
                        mma_ss(d_s, a, b, IDESC_QK, kk > 0 ? 1u : 0u);
                    }
                    tc_commit(&bar_s_full[(g + js) & 1]);
                    tc_commit(&bar_k_empty[st]);
                    if (js == w.n - 1) tc_commit(bar_q_empty);
                    gk++;
                    js++;
                    issued = true;
                }
            }
            if (jp < js) {
                const uint32_t gg = g + jp;
                const int buf = gg & 1;
                const int sv = gv % C::VS;
                if (jp == 0 && !o_free) o_free = mbar_test_wait(bar_o_empty, (it & 1) ^ 1);
                if ((jp > 0 || o_free) && mbar_test_wait(&bar_p_full[buf], (gg >> 1) & 1) &&
                    mbar_test_wait(&bar_v_full[sv], (gv / C::VS) & 1)) {
                    tc_fence_after();
                    const uint32_t a_tmem = tmem + C::S_COL0 + buf * 64;  // P occupies the first 32 columns of S
#pragma unroll
                    for (int kk = 0; kk < 4; kk++) {
                        const uint64_t b = dv0 + (uint64_t)((sv * C::KV_BYTES + kk * 2048) >> 4);
                        mma_ts(tmem + C::O_COL, a_tmem + kk * 8, b, IDESC_PV, (jp > 0 || kk > 0) ? 1u : 0u);
                    }
                    tc_commit(&bar_v_empty[sv]);
                    tc_commit(bar_o_done);
                    gv++;
                    jp++;
                    issued = true;
                }
            }
            if (issued) {
                waiting = false;
            } else if (!waiting) {
                t0 = clock64();
                waiting = true;
            } else if (*abort_flag || clock64() - t0 > p.timeout) {
                *abort_flag = 1;
                ok = false;
                break;
            }
        }
        if (!ok) break;
        g += w.n;
    }
    if (*abort_flag) {  // wait (bounded) for every MMA issued so far before TMEM is released
        tc_commit(bar_drain);
        volatile int never = 0;
        mbar_wait(bar_drain, 0, &never, 1ll << 26);
    }
}

// Copy of `nrows` finished output rows (from row `row0` of head offset `hb_off`)
// from this rank's output, read back from L2, to every other rank's output with
// lane-consecutive 16-byte stores (whole rows per warp instruction: the pattern
// that keeps NVLink writes in full lines).  One warp; nrows a multiple of the
// rows one instruction covers.
template <int D, bool BF16>
__device__ __forceinline__ void push_rows(const FwdParams& p, int64_t hb_off, int row0, int nrows) {
    using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
    constexpr int CPR = D / 8;     // 16-byte chunks per row
    constexpr int RPI = 32 / CPR;  // rows per warp instruction
    constexpr int BATCH = 8;
    const int lane = threadIdx.x & 31;
    const T* src = reinterpret_cast<const T*>(p.outs[p.rank]);
    const int r0 = row0 + lane / CPR;
    const int ni = nrows / RPI;  // instructions per destination
    // loads in batches ahead of their stores: the destinations could alias the
    // source as far as the compiler knows
#pragma unroll 1
    for (int i0 = 0; i0 < ni; i0 += BATCH) {
        uint4 v4[BATCH];
#pragma unroll
        for (int i = 0; i < BATCH; i++)
            if (i0 + i < ni)
                v4[i] = __ldcg(reinterpret_cast<const uint4*>(src + hb_off + (int64_t)(r0 + (i0 + i) * RPI) * p.o_sn) +
                               lane % CPR);
        for (int d = 0; d < p.n_out; d++) {
            if (d == p.rank) continue;
            T* dst = reinterpret_cast<T*>(p.outs[d]) + hb_off;
#pragma unroll
            for (int i = 0; i < BATCH; i++)
                if (i0 + i < ni)
                    *(reinterpret_cast<uint4*>(dst + (int64_t)(r0 + (i0 + i) * RPI) * p.o_sn) + lane % CPR) = v4[i];
        }
    }
}

// Fused all-gather, run by warp 3 while the softmax warps go on with the next
// item: each finished item's 128 output rows, already in this rank's output, go
// to every other rank (push_rows).  Items arrive through a two-slot ring; item
// -1 ends the loop.
template <int D, bool BF16>
__device__ void pusher(const FwdParams& p, uint64_t* bar_full, uint64_t* bar_empty, const int* push_item,
                       volatile int* abort_flag) {
    const int lane = threadIdx.x & 31;
    for (uint32_t k = 0;; k++) {
        const int ps = k & 1;
        if (!warp_wait(&bar_full[ps], (k >> 1) & 1, abort_flag, p.timeout)) return;
        const int item = push_item[ps];
        if (item < 0) return;
        const Item w = decode_item_n(p, item, 0);  // rows only
        push_rows<D, BF16>(p, (int64_t)w.b * p.o_sb + (int64_t)w.h * p.o_sh, w.qrow0, 128);
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar_empty[ps]);
    }
}

// Softmax warps' side of the ring: the warp's rows are in the output (fenced to
// GPU scope, so warp 3 reads them back from L2), then the item (or -1 to end)
// goes into the next slot once warp 3 has emptied it.
__device__ __forceinline__ bool enqueue_push(const FwdParams& p, uint64_t* bar_full, uint64_t* bar_empty,
                                             int* push_item, uint32_t& npush, int item, volatile int* abort_flag) {
    const int ps = npush & 1;
    if (!warp_wait(&bar_empty[ps], ((npush >> 1) & 1) ^ 1, abort_flag, p.timeout)) return false;
    __threadfence();
    if (threadIdx.x == 128) push_item[ps] = item;
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(&bar_full[ps]);
    npush++;
    return true;
}

// 32-byte global store (st.global.cs.v8.b32): one full sector per lane.
__device__ __forceinline__ void st_cs_v8(void* dst, const uint32_t* v) {
    asm volatile("st.global.cs.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(dst), "r"(v[0]), "r"(v[1]), "r"(v[2]),
                 "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
}

// The softmax warpgroup's view of a finished item whose output is still to be
// written (its epilogue runs after the next item's first step).
struct Pending {
    int item, n;       // the item (decoded again when its epilogue runs: fewer live registers)
    float m, l;
    uint32_t last_pv;  // global index of the item's last PV (o_done phase)
};

template <int D, bool BF16, int MODE>
__device__ void softmax_role(const FwdParams& p, uint32_t tmem, uint64_t* bar_item_full, uint64_t* bar_item_empty,
                             ItemSlot* slots, uint64_t* bar_s_full, uint64_t* bar_p_full, uint64_t* bar_o_done,
                             uint64_t* bar_o_empty, uint64_t* bar_wg, int* wg_flag, uint64_t* bar_push_full,
                             uint64_t* bar_push_empty, int* push_item, uint64_t* bar_final, volatile int* abort_flag) {
    using C = Cfg<D>;
    using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
    const int r = threadIdx.x - 128;  // query row within the tile == TMEM lane
    uint32_t npush = 0;               // items handed to the pusher (fused all-gather)
    uint32_t wg_uses = 0;             // phases of bar_wg (the 4 softmax warps) used so far
    const int lane = threadIdx.x & 31;
    const int half = r >> 6;
    const uint32_t t_lane = tmem + ((uint32_t)((r >> 5) * 32) << 16);
    const float sl2 = p.scale_log2;

    // Epilogue of a finished item: O / l -> the output (or, for a chunk of a
    // split global row, the chunk's unnormalised O with its m and l -> partial,
    // merged by the last chunk).  Waits for the item's last PV, whose o_done
    // phase is exact here: PV_{last-1} has completed (the next item's first S
    // was ready, and MMAs complete in issue order; on the way out it is waited
    // for explicitly) and the next PV needs this epilogue's o_empty first.  O's
    // TMEM is free for the next item's first PV once it returns.
    // Fused all-gather: a finished item's rows (in this rank's output) go to the
    // other ranks.  Items are handed to warp 3, which copies them while these
    // warps compute the next item; the CTA's final item, with nothing left to
    // compute, is copied by the four softmax warps themselves (each its own 32
    // rows), so the launch's tail is not one warp's copy of a whole item.
    auto hand_over = [&](int item, const Item& w, bool last) -> bool {
        if (!last) return enqueue_push(p, bar_push_full, bar_push_empty, push_item, npush, item, abort_flag);
        __threadfence();
        __syncwarp();
        push_rows<D, BF16>(p, (int64_t)w.b * p.o_sb + (int64_t)w.h * p.o_sh, w.qrow0 + (r & ~31), 32);
        return true;
    };
    auto finish = [&](const Pending& pd, bool last) -> bool {
        const Item w = decode_item_n(p, pd.item, pd.n);
        if (!warp_wait(bar_o_done, pd.last_pv & 1, abort_flag, p.timeout)) return false;
        tc_fence_after();
        int orow = w.qrow0 + r;  // output token row of this thread's query
        if constexpr (MODE == MODE_ROWS) orow = p.row_map[orow];
        if constexpr (MODE == MODE_SQUARES) {
            const int blk = orow >> 6;
            if (blk >= p.text_blocks) {  // tile row r%64 of an image block = row-major position in its square
                const int o = square_origin(p, blk - p.text_blocks);
                orow = o < 0 ? -1 : 64 * p.text_blocks + o + ((orow & 63) >> 3) * p.grid + (orow & 7);
            }
        }
        const bool row_ok = orow >= 0 && orow < p.N;  // a bad map entry drops the row, never stores out of range
        const int64_t ooff = (int64_t)w.b * p.o_sb + (int64_t)w.h * p.o_sh + (int64_t)(row_ok ? orow : 0) * p.o_sn;
        // every destination has the same address residue mod 32 (checked on the host)
        const uintptr_t addr0 = reinterpret_cast<uintptr_t>(reinterpret_cast<T*>(p.outs[0]) + ooff);
        const bool vec = (addr0 & 15) == 0, vec32 = (addr0 & 31) == 0;
        // Rows are written to this rank's output first (lane = row); in the fused
        // all-gather the item is then handed to warp 3 (pusher), which copies the
        // rows to the other ranks while this warp goes on.
        const bool push = p.n_out > 1 && vec;
        auto store32 = [&](int c0, const uint32_t (&packed)[16]) {  // 32 output columns, packed 16-bit pairs
            for (int d = 0; d < p.n_out && row_ok; d++) {
                if (d != p.rank && push) continue;
                T* orow_p = reinterpret_cast<T*>(p.outs[d]) + ooff + c0;
                if (vec32) {  // written once, read by the next layer: do not keep in L2 over K/V
                    st_cs_v8(orow_p, packed);
                    st_cs_v8(orow_p + 16, packed + 8);
                } else if (vec) {
                    uint4* dst = reinterpret_cast<uint4*>(orow_p);
#pragma unroll
                    for (int i = 0; i < 4; i++)
                        __stcs(dst + i, make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]));
                } else {
                    uint16_t* dst = reinterpret_cast<uint16_t*>(orow_p);
#pragma unroll
                    for (int i = 0; i < 16; i++) {
                        dst[2 * i] = (uint16_t)(packed[i] & 0xffffu);
                        dst[2 * i + 1] = (uint16_t)(packed[i] >> 16);
                    }
                }
            }
        };
        if (!w.split) {
            const float inv = 1.f / pd.l;
#pragma unroll
            for (int c = 0; c < D / 32; c++) {
                uint32_t o[32];
                tmem_ld32(t_lane + C::O_COL + 32 * c, o);
                uint32_t packed[16];
#pragma unroll
                for (int i = 0; i < 16; i++)
                    packed[i] = pack2<BF16>(__uint_as_float(o[2 * i]) * inv, __uint_as_float(o[2 * i + 1]) * inv);
                store32(32 * c, packed);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_o_empty);
            if (push && !hand_over(pd.item, w, last)) return false;
        } else {
            // a chunk's record: O as float4 groups of 4 columns, group-major
            // ([D/4][128 rows][4]), so the 32 rows of a warp fill 512 contiguous bytes
            // per store (and per load in the merge); then m [128] and l [128]
            constexpr int PSTRIDE = 128 * D + 256;
            float* rec = p.partial + ((int64_t)w.group * p.n_chunks + w.chunk) * PSTRIDE;
            float4* rec4 = reinterpret_cast<float4*>(rec);
#pragma unroll
            for (int c = 0; c < D / 32; c++) {
                uint32_t o[32];
                tmem_ld32(t_lane + C::O_COL + 32 * c, o);
#pragma unroll
                for (int i = 0; i < 8; i++)
                    rec4[(8 * c + i) * 128 + r] = make_float4(__uint_as_float(o[4 * i]), __uint_as_float(o[4 * i + 1]),
                                                              __uint_as_float(o[4 * i + 2]), __uint_as_float(o[4 * i + 3]));
            }
            rec[128 * D + r] = pd.m;
            rec[128 * D + 128 + r] = pd.l;
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_o_empty);  // O's TMEM may be reused now
            __threadfence();                          // partial visible before the count below
            // all 128 rows written -> count this chunk; the last chunk of the row merges
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_wg);
            if (!warp_wait(bar_wg, wg_uses & 1, abort_flag, p.timeout)) return false;
            wg_uses++;
            if (r == 0) {
                const int done = atomicAdd(&p.chunk_cnt[w.group], 1);
                const int last = done == p.n_chunks - 1;
                if (last) p.chunk_cnt[w.group] = 0;  // ready for the next launch
                *wg_flag = last;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_wg);
            if (!warp_wait(bar_wg, wg_uses & 1, abort_flag, p.timeout)) return false;
            wg_uses++;
            if (*wg_flag) {
                __threadfence();
                const float* base = p.partial + (int64_t)w.group * p.n_chunks * PSTRIDE;
                // chunk weights 2^(m_c - max) are recomputed where used (no
                // indexed local array, which would live in local memory)
                float mmax = -INFINITY;
                for (int c = 0; c < p.n_chunks; c++) mmax = fmaxf(mmax, __ldcg(base + c * PSTRIDE + 128 * D + r));
                auto weight = [&](int c) {
                    const float mc = __ldcg(base + c * PSTRIDE + 128 * D + r);
                    return mc == -INFINITY ? 0.f : ex2(mc - mmax);
                };
                float lsum = 0.f;
                for (int c = 0; c < p.n_chunks; c++) lsum += weight(c) * __ldcg(base + c * PSTRIDE + 128 * D + 128 + r);
                const float inv = 1.f / lsum;
                for (int c = 0; c < D / 32; c++) {
                    float vals[32];
#pragma unroll
                    for (int i = 0; i < 32; i++) vals[i] = 0.f;
                    for (int k = 0; k < p.n_chunks; k++) {
                        const float wk = weight(k);
                        const float4* src = reinterpret_cast<const float4*>(base + k * PSTRIDE);
#pragma unroll
                        for (int i = 0; i < 8; i++) {
                            const float4 v4 = __ldcg(src + (8 * c + i) * 128 + r);
                            vals[4 * i] += wk * v4.x;
                            vals[4 * i + 1] += wk * v4.y;
                            vals[4 * i + 2] += wk * v4.z;
                            vals[4 * i + 3] += wk * v4.w;
                        }
                    }
                    uint32_t packed[16];
#pragma unroll
                    for (int i = 0; i < 16; i++) packed[i] = pack2<BF16>(vals[2 * i] * inv, vals[2 * i + 1] * inv);
                    store32(32 * c, packed);
                }
                if (push && !hand_over(pd.item, w, last)) return false;
            }
        }
        return true;
    };

    Pending pend;
    bool pending = false;
    uint32_t g = 0;
    for (int it = 0;; it++) {
        const int slot = it & 1;
        if (!warp_wait(&bar_item_full[slot], (it >> 1) & 1, abort_flag, p.timeout)) return;
        const int item = slots[slot].item;
        const int n_item = slots[slot].n;
        int chunk = slots[slot].flags[lane];  // lane l: flags of entry l
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar_item_empty[slot]);
        if (item >= p.num_items) {
            // No later S was waited for: wait until every MMA of this CTA has
            // completed (the issuer's final commit), then finish() finds the
            // last PV's o_done phase complete and no later one.
            if (pending && !warp_wait(bar_final, 0, abort_flag, p.timeout)) return;
            if (pending && !finish(pend, true)) return;
            if (p.n_out > 1) enqueue_push(p, bar_push_full, bar_push_empty, push_item, npush, -1, abort_flag);
            return;
        }
        const Item w = decode_item_n(p, item, n_item);
        float m = -INFINITY, l = 0.f;
        int next_chunk = 0;
        // one softmax step: scores S_j -> P_j (and the running max / sum)
        auto step = [&](int j) -> bool {
            const uint32_t gg = g + j;
            const int buf = gg & 1;
            if (!w.global) {
                if ((j & 31) == 0 && j > 0) chunk = next_chunk;
                if ((j & 31) == 16 && j + 16 < w.n) {  // flags of entries j+16 .. j+47, a step ahead of use
                    const int jj = j + 16 + lane;
                    next_chunk = jj < w.n ? p.flags[(int64_t)w.row * p.W + jj] : 0;
                }
            }
            const int fl = w.global ? 3 : __shfl_sync(FULL, chunk, j & 31);
            const bool allowed = (fl >> half) & 1;  // uniform per warp
            if (!warp_wait(&bar_s_full[buf], (gg >> 1) & 1, abort_flag, p.timeout)) return false;
            tc_fence_after();
            const uint32_t s_addr = t_lane + C::S_COL0 + buf * 64;
            uint32_t pk[32];
            float m_new = m, alpha = 1.f;
            if (allowed) {
                uint32_t s_[64];
                tmem_ld64(s_addr, s_);
                // row max: 3-input max over four independent chains
                float a0 = fmaxf(__uint_as_float(s_[0]), __uint_as_float(s_[1]));
                float a1 = fmaxf(__uint_as_float(s_[2]), __uint_as_float(s_[3]));
                float a2 = fmaxf(__uint_as_float(s_[4]), __uint_as_float(s_[5]));
                float a3 = fmaxf(__uint_as_float(s_[6]), __uint_as_float(s_[7]));
#pragma unroll
                for (int i = 8; i < 64; i += 8) {
                    a0 = fmax3(a0, __uint_as_float(s_[i]), __uint_as_float(s_[i + 1]));
                    a1 = fmax3(a1, __uint_as_float(s_[i + 2]), __uint_as_float(s_[i + 3]));
                    a2 = fmax3(a2, __uint_as_float(s_[i + 4]), __uint_as_float(s_[i + 5]));
                    a3 = fmax3(a3, __uint_as_float(s_[i + 6]), __uint_as_float(s_[i + 7]));
                }
                const float mx = fmaxf(fmax3(a0, a1, a2), a3) * sl2;
                if (mx > m + RESCALE_THRESHOLD) {
                    m_new = mx;
                    alpha = ex2(m - m_new);  // 0 when m == -inf
                }
                // p = 2^(s*scale*log2e - m): packed FMA for the argument, MUFU ex2,
                // packed adds into four partial row sums
                const uint64_t scale2 = f2_pack(sl2, sl2);
                const uint64_t neg_m2 = f2_pack(-m_new, -m_new);
                uint64_t acc[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
                for (int i = 0; i < 32; i++) {
                    const uint64_t x2 = f2_fma(f2_pack(__uint_as_float(s_[2 * i]), __uint_as_float(s_[2 * i + 1])),
                                               scale2, neg_m2);
                    float x0, x1;
                    f2_unpack(x2, x0, x1);
                    const float p0 = ex2(x0), p1 = ex2(x1);
                    acc[i & 3] = f2_add(acc[i & 3], f2_pack(p0, p1));
                    pk[i] = pack2<BF16>(p0, p1);
                }
                float s0, s1, s2, s3;
                f2_unpack(f2_add(acc[0], acc[1]), s0, s1);
                f2_unpack(f2_add(acc[2], acc[3]), s2, s3);
                l = l * alpha + ((s0 + s1) + (s2 + s3));
            } else {
#pragma unroll
                for (int i = 0; i < 32; i++) pk[i] = 0u;
            }
            tmem_st32(s_addr, pk);
            // O may only be rescaled once PV_{gg-1} has completed.  S_gg being ready
            // means PV_{gg-2} completed (it was issued first), and PV_gg waits for
            // this step's P, so o_done is at phase gg-1 or gg: waiting on the parity
            // of gg-1 is exact without having waited the earlier phases.  Only a
            // rescale needs that wait (step 0 of an item never rescales).
            const bool need = (m_new != m) && (m != -INFINITY);
            const bool rescale = __any_sync(FULL, need);
            if (rescale) {
                if (!warp_wait(bar_o_done, (gg - 1) & 1, abort_flag, p.timeout)) return false;
                tc_fence_after();
                const float a = need ? alpha : 1.f;
#pragma unroll
                for (int c = 0; c < D / 32; c++) {
                    uint32_t o[32];
                    tmem_ld32(t_lane + C::O_COL + 32 * c, o);
#pragma unroll
                    for (int i = 0; i < 32; i++) o[i] = __float_as_uint(__uint_as_float(o[i]) * a);
                    tmem_st32(t_lane + C::O_COL + 32 * c, o);
                }
            }
            m = m_new;
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar_p_full[buf]);
            return true;
        };
        // step 0, then the previous item's epilogue (after this item's first P is
        // handed over: its last PV has had a step to complete, and this item's
        // first PV, which needs O's TMEM, follows right after), then the rest
        if (!step(0)) return;
        if (pending) {
            if (!finish(pend, false)) return;
            pending = false;
        }
        for (int j = 1; j < w.n; j++)
            if (!step(j)) return;
        pend.n = w.n;
        pend.item = item;
        pend.m = m;
        pend.l = l;
        pend.last_pv = g + w.n - 1;
        pending = true;
        g += w.n;
    }
}

// Fused all-gather completion, run by one thread after every CTA of the launch
// has stored its rows and fenced them at system scope: publish this rank's
// epoch to every rank, then wait (bounded) for every rank's epoch here.
__device__ __noinline__ void peer_complete(const FwdParams& p) {
    __threadfence_system();
    for (int i = 0; i < p.n_out; i++) st_release_sys(p.peer_flags[i] + p.rank, p.epoch);
    const int32_t* mine = p.peer_flags[p.rank];
    const long long t0 = clock64();
    for (int i = 0; i < p.n_out; i++) {
        // epochs only grow: compare by wrap-safe difference
        while ((int32_t)((uint32_t)ld_acquire_sys(mine + i) - (uint32_t)p.epoch) < 0) {
            if (clock64() - t0 > p.peer_timeout) {
                atomicOr(&p.ws[2], HB_DEV_PEER_TIMEOUT);
                return;
            }
        }
    }
}

template <int D, bool BF16, int MODE>
__global__ void __launch_bounds__(256, 2) k_paired_fwd(const __grid_constant__ FwdParams p) {
    using C = Cfg<D>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // The 128-byte swizzle of the tiles assumes 1024-byte aligned tile bases; the
    // region has no static shared memory before it, so this holds, and is checked.
    if (smem_u32(smem_raw) & 1023) {
        if (threadIdx.x == 0) atomicOr(&p.ws[2], HB_DEV_SMEM_ALIGN);
        return;
    }
    uint8_t* sQ = smem_raw;
    uint8_t* sK = sQ + C::Q_BYTES;
    uint8_t* sV = sK + C::KS * C::KV_BYTES;
    typename C::Ctl* ctl = reinterpret_cast<typename C::Ctl*>(smem_raw + C::CTL_OFF);
    uint64_t &bar_q_full = ctl->q_full, &bar_q_empty = ctl->q_empty, &bar_o_done = ctl->o_done;
    uint64_t &bar_o_empty = ctl->o_empty, &bar_drain = ctl->drain, &bar_wg = ctl->wg;
    uint64_t *bar_k_full = ctl->k_full, *bar_k_empty = ctl->k_empty;
    uint64_t *bar_v_full = ctl->v_full, *bar_v_empty = ctl->v_empty;
    uint64_t *bar_s_full = ctl->s_full, *bar_p_full = ctl->p_full;
    uint64_t *bar_item_full = ctl->item_full, *bar_item_empty = ctl->item_empty;
    ItemSlot* slots = ctl->slots;
    uint32_t& tmem_base_sh = ctl->tmem_base;
    int& abort_sh = ctl->abort;
    int& wg_flag = ctl->wg_flag;
    volatile int* abort_flag = &abort_sh;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        mbar_init(&bar_q_full, 1);
        mbar_init(&bar_q_empty, 1);
        mbar_init(&bar_o_done, 1);
        mbar_init(&bar_o_empty, 4);
        mbar_init(&bar_drain, 1);
        mbar_init(&ctl->final_done, 1);
        mbar_init(&bar_wg, 4);
        for (int i = 0; i < C::KS; i++) {
            mbar_init(&bar_k_full[i], 1);
            mbar_init(&bar_k_empty[i], 1);
        }
        for (int i = 0; i < C::VS; i++) {
            mbar_init(&bar_v_full[i], 1);
            mbar_init(&bar_v_empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&bar_s_full[i], 1);
            mbar_init(&bar_p_full[i], 4);
            mbar_init(&bar_item_full[i], 1);
            mbar_init(&bar_item_empty[i], 6);  // V producer, MMA issuer, 4 softmax warps
            mbar_init(&ctl->push_full[i], 4);
            mbar_init(&ctl->push_empty[i], 1);
        }
        abort_sh = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&p.tmap_q);
        prefetch_tmap(&p.tmap_k);
        prefetch_tmap(&p.tmap_v);
    }
    if (warp == 3) {
        tmem_alloc(&tmem_base_sh, C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_sh;

    if (warp == 0) {
        producer<D, 0, MODE>(p, sQ, sK, bar_item_full, bar_item_empty, slots, &bar_q_full, &bar_q_empty, bar_k_full,
                       bar_k_empty, abort_flag);
    } else if (warp == 1) {
        producer<D, 1, MODE>(p, sQ, sV, bar_item_full, bar_item_empty, slots, &bar_q_full, &bar_q_empty, bar_v_full,
                       bar_v_empty, abort_flag);
    } else if (warp == 2) {
        if (lane == 0)
            mma_issuer<D, BF16>(p, tmem, sQ, sK, sV, bar_item_full, bar_item_empty, slots, &bar_q_full,
                                &bar_q_empty, bar_k_full, bar_k_empty, bar_v_full, bar_v_empty, bar_s_full, bar_p_full,
                                &bar_o_done, &bar_o_empty, &bar_drain, &ctl->final_done, abort_flag);
    } else if (warp >= 4) {
        softmax_role<D, BF16, MODE>(p, tmem, bar_item_full, bar_item_empty, slots, bar_s_full, bar_p_full, &bar_o_done,
                              &bar_o_empty, &bar_wg, &wg_flag, ctl->push_full, ctl->push_empty, ctl->push_item,
                              &ctl->final_done, abort_flag);
    } else if (warp == 3 && p.n_out > 1) {
        pusher<D, BF16>(p, ctl->push_full, ctl->push_empty, ctl->push_item, abort_flag);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 3) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
    if (threadIdx.x == 0) {
        if (abort_sh) atomicOr(&p.ws[2], HB_DEV_TIMEOUT);
        // The CTA's row stores (all threads, ordered before this thread by the
        // barrier above) are made visible at the scope the consumers need before
        // the CTA is counted: one fence per CTA (a system-scope fence in every
        // thread costs milliseconds per launch).
        if (p.n_out > 1)
            __threadfence_system();
        else
            __threadfence();
        const int prev = atomicAdd(&p.ws[1], 1);
        if (prev == (int)gridDim.x - 1) {  // last CTA: reset the work counter for the next launch
            atomicExch(&p.ws[0], 0);
            atomicExch(&p.ws[1], 0);
            __threadfence();
            if (p.n_out > 1) peer_complete(p);
        }
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    });
    return fn;
}

// [B][H][N][D] view with element strides (sb, sh, sn), D contiguous -> 4-D tiled
// map (d, then n/h/b sorted by stride), box = 64 x box_rows, 128-byte swizzle.
int make_tmap(CUtensorMap* map, const void* base, bool bf16, int D, int N, int H, int B, int64_t sb, int64_t sh,
              int64_t sn, int box_rows, int32_t perm[3]) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return HB_ERR_CUDA;
    if (reinterpret_cast<uintptr_t>(base) & 15) return HB_ERR_TMA;
    const int64_t ext[3] = {N, H, B};
    int64_t strideb[3] = {sn * 2, sh * 2, sb * 2};
    int64_t span = (int64_t)D * 2;
    for (int i = 0; i < 3; i++)
        if (ext[i] > 1) span = std::max<int64_t>(span, ext[i] * strideb[i]);
    for (int i = 0; i < 3; i++) {
        if (ext[i] == 1) strideb[i] = (span + 15) & ~int64_t(15);  // never used for addressing
        if (strideb[i] <= 0 || (strideb[i] & 15) || strideb[i] >= (int64_t(1) << 40)) return HB_ERR_TMA;
    }
    int order[3] = {0, 1, 2};
    for (int a = 0; a < 3; a++)
        for (int b = a + 1; b < 3; b++)
            if (strideb[order[b]] < strideb[order[a]] ||
                (strideb[order[b]] == strideb[order[a]] && order[b] < order[a]))
                std::swap(order[a], order[b]);
    cuuint64_t gdim[4], gstride[3];
    cuuint32_t box[4], estride[4] = {1, 1, 1, 1};
    gdim[0] = (cuuint64_t)D;
    box[0] = 64;
    for (int k = 0; k < 3; k++) {
        const int dim = order[k];
        gdim[k + 1] = (cuuint64_t)ext[dim];
        gstride[k] = (cuuint64_t)strideb[dim];
        box[k + 1] = dim == 0 ? (cuuint32_t)box_rows : 1u;
        perm[dim] = k + 1;
    }
    const CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                           const_cast<void*>(base), gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? HB_OK : HB_ERR_TMA;
}

// Gather mode: the tensor as 2-D (D, rows) with a one-row box, where row
// b*rs[0] + h*rs[1] + n*rs[2] holds token n of head h, batch b.  Needs every
// outer stride to be a multiple of D (rows of D contiguous elements).
int make_tmap_rows(CUtensorMap* map, const void* base, bool bf16, int D, int N, int H, int B, int64_t sb, int64_t sh,
                   int64_t sn, int64_t rs[3]) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return HB_ERR_CUDA;
    if (reinterpret_cast<uintptr_t>(base) & 15) return HB_ERR_TMA;
    const int64_t ext[3] = {B, H, N}, st[3] = {sb, sh, sn};
    int64_t rows = 1;
    for (int i = 0; i < 3; i++) {
        if (ext[i] == 1) {
            rs[i] = 0;
            continue;
        }
        if (st[i] <= 0 || st[i] % D) return HB_ERR_TMA;
        rs[i] = st[i] / D;
        rows += (ext[i] - 1) * rs[i];
    }
    if (rows >= INT32_MAX) return HB_ERR_UNSUPPORTED;
    cuuint64_t gdim[2] = {(cuuint64_t)D, (cuuint64_t)rows};
    cuuint64_t gstride[1] = {(cuuint64_t)D * 2};
    cuuint32_t box[2] = {64, 1}, estride[2] = {1, 1};
    const CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                           const_cast<void*>(base), gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? HB_OK : HB_ERR_TMA;
}

// MODE_SQUARES image map: the g x g image tokens that follow `text` tokens, as
// (D, x, y, head, batch) with element strides (1, sn, g*sn, sh, sb) and a
// {64, 8, 8, 1, 1} box, so one load gives an aligned 8x8 square as 64 swizzled
// 128-byte rows in row-major square order.
int make_tmap_img(CUtensorMap* map, const void* base, bool bf16, int D, int text, int g, int H, int B, int64_t sb,
                  int64_t sh, int64_t sn) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return HB_ERR_CUDA;
    const char* img = static_cast<const char*>(base) + (int64_t)text * sn * 2;
    if (reinterpret_cast<uintptr_t>(img) & 15) return HB_ERR_TMA;
    int64_t st[4] = {sn * 2, (int64_t)g * sn * 2, sh * 2, sb * 2};
    const int64_t ext[4] = {g, g, H, B};
    for (int i = 0; i < 4; i++) {
        if (ext[i] == 1) st[i] = 16;  // never used for addressing
        if (st[i] <= 0 || (st[i] & 15) || st[i] >= (int64_t(1) << 40)) return HB_ERR_TMA;
    }
    cuuint64_t gdim[5] = {(cuuint64_t)D, (cuuint64_t)g, (cuuint64_t)g, (cuuint64_t)H, (cuuint64_t)B};
    cuuint64_t gstride[4] = {(cuuint64_t)st[0], (cuuint64_t)st[1], (cuuint64_t)st[2], (cuuint64_t)st[3]};
    cuuint32_t box[5] = {64, 8, 8, 1, 1}, estride[5] = {1, 1, 1, 1, 1};
    const CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5,
                           const_cast<char*>(img), gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? HB_OK : HB_ERR_TMA;
}

struct DeviceInfo {
    int sms = 0;
    int clock_khz = 0;
    bool configured[12] = {};
};
std::mutex g_mu;
DeviceInfo g_dev[64];

// SM count and SM clock of a device, queried once (the attribute queries are
// not free, and the launch path runs once per attention call).
int device_info(int dev, int* sms, int* clock_khz) {
    std::lock_guard<std::mutex> lk(g_mu);
    DeviceInfo& di = g_dev[dev];
    if (!di.sms) {
        HB_CUDA_TRY(cudaDeviceGetAttribute(&di.clock_khz, cudaDevAttrClockRate, dev));
        HB_CUDA_TRY(cudaDeviceGetAttribute(&di.sms, cudaDevAttrMultiProcessorCount, dev));
    }
    if (sms) *sms = di.sms;
    if (clock_khz) *clock_khz = di.clock_khz;
    return HB_OK;
}

template <int D, bool BF16, int MODE>
int launch(const FwdParams& p, int dev, cudaStream_t st) {
    using C = Cfg<D>;
    auto kern = k_paired_fwd<D, BF16, MODE>;
    const int slot = (D == 128 ? 2 : 0) + (BF16 ? 1 : 0) + 4 * MODE;
    int sms, rc;
    if ((rc = device_info(dev, &sms, nullptr))) return rc;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        DeviceInfo& di = g_dev[dev];
        if (!di.configured[slot]) {
            HB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
            di.configured[slot] = true;
        }
    }
    const int grid = std::min(p.num_items, 2 * sms);
    kern<<<grid, 256, C::SMEM, st>>>(p);
    HB_LAUNCH_CHECK();
    return HB_OK;
}

}  // namespace
}  // namespace hb

using namespace hb;

namespace hb {
namespace {
// How the global pair-rows split over their key blocks: chunks of ~CHUNK_BLOCKS
// blocks (at most MAX_CHUNKS), and the workspace bytes that split needs.
struct SplitPlan {
    int chunk, n_chunks;
    int64_t partial_bytes, bytes;  // bytes: smallest workspace that fits the partials
};
SplitPlan split_plan(int B, int H, int N, int G, int D) {
    SplitPlan s;
    const int nkb = N / 64;
    s.chunk = std::max(CHUNK_BLOCKS, (nkb + MAX_CHUNKS - 1) / MAX_CHUNKS);
    s.n_chunks = (nkb + s.chunk - 1) / s.chunk;
    const int64_t groups = (int64_t)B * H * (G / 128);
    s.partial_bytes = groups * s.n_chunks * (int64_t)(128 * D + 256) * 4;
    if (groups == 0 || s.n_chunks <= 1) {
        s.n_chunks = 1;
        s.chunk = nkb;
        s.partial_bytes = 0;
        s.bytes = WS_HEADER;
        return s;
    }
    // Smallest size with 256 bytes to spare over header + counters + partials;
    // the spare keeps every larger size fitting too (the counter region grows
    // by 256 bytes per ~4 MB of workspace).
    int64_t w = WS_HEADER + s.partial_bytes;
    while (w < WS_HEADER + counter_bytes(w) + s.partial_bytes + 256) w = WS_HEADER + counter_bytes(w) + s.partial_bytes + 256;
    s.bytes = w;
    return s;
}
inline bool split_fits(const SplitPlan& s, int64_t ws) {
    return s.partial_bytes > 0 && ws - WS_HEADER - counter_bytes(ws) >= s.partial_bytes;
}
}  // namespace
}  // namespace hb

extern "C" size_t hb_fwd_workspace_bytes(void) { return 64; }

extern "C" size_t hb_fwd_workspace_bytes_for(int B, int H, int N, int G, int D) {
    if (B <= 0 || H <= 0 || N <= 0 || N % 128 || G < 0 || G % 128 || G >= N || (D != 64 && D != 128)) return 0;
    return (size_t)std::max<int64_t>(WS_HEADER, split_plan(B, H, N, G, D).bytes);
}

namespace hb {
namespace {
// Shared body of hb_paired_fwd (out, optional row_map) and hb_paired_fwd_allgather
// (peers: every rank's output and flag words).
int paired_fwd(const void* q, const void* k, const void* v, void* out, const int64_t* strides, int B, int H, int N,
               int D, int G, int W, int key_block_size, const int32_t* kv_indices, const int32_t* kv_flags,
               const int32_t* kv_counts, float scale_log2, int dtype, const int32_t* row_map,
               const hb_raster_order_t* raster, const hb_peer_out_t* peers, void* workspace, size_t workspace_bytes,
               void* stream_) {
    if (!q || !k || !v || !(out || peers) || !strides || !workspace) return HB_ERR_ARG;
    if (raster) {
        const int64_t T = raster->text_tokens, g = raster->grid;
        if (T < 0 || T % 64 || g <= 0 || g % 8 || T + g * g != (int64_t)N || !raster->block_origin ||
            (reinterpret_cast<uintptr_t>(raster->block_origin) & 3) || row_map || peers)
            return HB_ERR_ARG;
    }
    if (peers) {
        const int n = peers->n_ranks;
        if (n < 1 || n > HB_MAX_RANKS || peers->rank < 0 || peers->rank >= n || peers->epoch <= 0 ||
            peers->timeout_ms < 0)
            return HB_ERR_ARG;
        for (int i = 0; i < n; i++) {
            if (!peers->out[i] || !peers->flags[i] || (reinterpret_cast<uintptr_t>(peers->flags[i]) & 3))
                return HB_ERR_ARG;
            if (reinterpret_cast<uintptr_t>(peers->out[i]) & 15) return HB_ERR_ARG;  // 16-byte row stores
        }
        if (strides[9] % 8 || strides[10] % 8 || strides[11] % 8) return HB_ERR_ARG;
    }
    if (row_map && (reinterpret_cast<uintptr_t>(row_map) & 15)) return HB_ERR_ARG;
    if (workspace_bytes < hb_fwd_workspace_bytes() || (reinterpret_cast<uintptr_t>(workspace) & 255))
        return HB_ERR_WORKSPACE;
    if (B <= 0 || H <= 0 || N <= 0 || N % 128 || G < 0 || G % 128 || G >= N || W < 1) return HB_ERR_ARG;
    if (D != 64 && D != 128) return HB_ERR_UNSUPPORTED;
    if (key_block_size != 64) return HB_ERR_UNSUPPORTED;
    if (dtype != 0 && dtype != 1) return HB_ERR_UNSUPPORTED;
    if (!(scale_log2 > 0.f) || scale_log2 == INFINITY) return HB_ERR_ARG;
    const int o_rows = (N - G) / 128;
    if (o_rows > 0 && (!kv_indices || !kv_flags || !kv_counts)) return HB_ERR_ARG;
    const int64_t items = (int64_t)B * H * (N / 128);
    if (items > INT32_MAX / 2) return HB_ERR_UNSUPPORTED;
    int dev;
    HB_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return HB_ERR_UNSUPPORTED;

    FwdParams p;
    memset(&p, 0, sizeof(p));
    const bool bf16 = dtype == 1;
    int rc;
    if (row_map) {
        p.row_map = row_map;
        if ((rc = make_tmap_rows(&p.tmap_q, q, bf16, D, N, H, B, strides[0], strides[1], strides[2], p.rs_q))) return rc;
        if ((rc = make_tmap_rows(&p.tmap_k, k, bf16, D, N, H, B, strides[3], strides[4], strides[5], p.rs_k))) return rc;
        if ((rc = make_tmap_rows(&p.tmap_v, v, bf16, D, N, H, B, strides[6], strides[7], strides[8], p.rs_v))) return rc;
    } else if (raster) {
        if ((rc = make_tmap(&p.tmap_q, q, bf16, D, N, H, B, strides[0], strides[1], strides[2], 64, p.perm_q))) return rc;
        if ((rc = make_tmap(&p.tmap_k, k, bf16, D, N, H, B, strides[3], strides[4], strides[5], 64, p.perm_k))) return rc;
        if ((rc = make_tmap(&p.tmap_v, v, bf16, D, N, H, B, strides[6], strides[7], strides[8], 64, p.perm_v))) return rc;
        const int T = raster->text_tokens, g = raster->grid;
        if ((rc = make_tmap_img(&p.tmap_q_img, q, bf16, D, T, g, H, B, strides[0], strides[1], strides[2]))) return rc;
        if ((rc = make_tmap_img(&p.tmap_k_img, k, bf16, D, T, g, H, B, strides[3], strides[4], strides[5]))) return rc;
        if ((rc = make_tmap_img(&p.tmap_v_img, v, bf16, D, T, g, H, B, strides[6], strides[7], strides[8]))) return rc;
        p.text_blocks = T / 64;
        p.grid = g;
        p.img_blocks = g * g / 64;
        p.sq_origin = raster->block_origin;
    } else {
        if ((rc = make_tmap(&p.tmap_q, q, bf16, D, N, H, B, strides[0], strides[1], strides[2], 128, p.perm_q))) return rc;
        if ((rc = make_tmap(&p.tmap_k, k, bf16, D, N, H, B, strides[3], strides[4], strides[5], 64, p.perm_k))) return rc;
        if ((rc = make_tmap(&p.tmap_v, v, bf16, D, N, H, B, strides[6], strides[7], strides[8], 64, p.perm_v))) return rc;
    }
    if (peers) {
        const int n = peers->n_ranks;
        for (int i = 0; i < n; i++) {
            p.outs[i] = peers->out[i];
            p.peer_flags[i] = peers->flags[i];
        }
        p.n_out = n;
        p.rank = peers->rank;
        p.epoch = peers->epoch;
        int khz = 0;
        if ((rc = device_info(dev, nullptr, &khz))) return rc;
        const long long ms = peers->timeout_ms ? peers->timeout_ms : 10000;
        p.peer_timeout = ms * (long long)(khz > 0 ? khz : 2000000);
    } else {
        p.outs[0] = out;
        p.n_out = 1;
    }
    p.o_sb = strides[9];
    p.o_sh = strides[10];
    p.o_sn = strides[11];
    p.indices = kv_indices;
    p.flags = kv_flags;
    p.counts = kv_counts;
    p.ws = reinterpret_cast<int32_t*>(workspace);
    p.B = B;
    p.H = H;
    p.N = N;
    p.G = G;
    p.W = W;
    p.g_rows = G / 128;
    p.o_rows = o_rows;
    p.nkb = N / 64;
    // Split the global pair-rows (every key block) only when one of them would
    // outlast a CTA's share of the work (est. from the metadata width W; two CTAs
    // per SM), and only when the caller's workspace holds the partials.
    const SplitPlan sp = split_plan(B, H, N, G, D);
    int n_chunks = 1;
    if (sp.n_chunks > 1 && split_fits(sp, (int64_t)workspace_bytes)) {
        int sms = 0;
        if ((rc = device_info(dev, &sms, nullptr))) return rc;
        const double share = (double)B * H * ((double)p.g_rows * p.nkb + (double)o_rows * W) / (2.0 * sms);
        const int target = std::max(CHUNK_BLOCKS, (int)(0.75 * share));
        n_chunks = std::min(sp.n_chunks, (p.nkb + target - 1) / target);
    }
    // No even split (long global rows are no longer than a CTA's share here):
    // keep each global row whole but for TAIL_CHUNKS chunks of half an ordinary
    // pair-row, scheduled after every ordinary row, so the launch ends on short
    // items.  Only for wide rows (W / 2 >= CHUNK_BLOCKS: the tail the CTAs leave
    // grows with the item length, the split's partials and merge do not):
    // measured 1-2 % faster at 2048^2 t4k1 and 4096^2 t16k3 (W = 75), 3 % slower
    // at 2048^2 t16k3 (W = 27).  Needs the workspace to hold the partials.
    int tail_chunks = 0, tail_blocks = 0;
    if (n_chunks == 1 && p.g_rows > 0 && W / 2 >= CHUNK_BLOCKS) {
        tail_blocks = W / 2;
        const int64_t need = (int64_t)B * H * p.g_rows * (1 + TAIL_CHUNKS) * (int64_t)(128 * D + 256) * 4;
        const int64_t ws = (int64_t)workspace_bytes;
        if (p.nkb >= TAIL_CHUNKS * tail_blocks + CHUNK_BLOCKS && ws - WS_HEADER - counter_bytes(ws) >= need)
            tail_chunks = TAIL_CHUNKS;
    }
    p.head_chunks = n_chunks;
    p.tail_chunks = tail_chunks;
    p.tail_blocks = tail_blocks;
    p.head_blocks = p.nkb - tail_chunks * tail_blocks;
    p.n_chunks = n_chunks + tail_chunks;
    p.chunk = (p.head_blocks + n_chunks - 1) / n_chunks;
    const bool split = p.n_chunks > 1;
    if (split) {
        p.chunk_cnt = reinterpret_cast<int32_t*>(reinterpret_cast<char*>(workspace) + WS_HEADER);
        p.partial = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + WS_HEADER +
                                             counter_bytes((int64_t)workspace_bytes));
    }
    p.n_global_items = B * H * p.g_rows * p.head_chunks;
    p.n_ordinary_items = B * H * o_rows;
    p.num_items = p.n_global_items + p.n_ordinary_items + B * H * p.g_rows * p.tail_chunks;
    p.scale_log2 = scale_log2;
    p.timeout = 2000000000ll;
    cudaStream_t st = (cudaStream_t)stream_;
    if (row_map) {
        if (D == 128) return bf16 ? launch<128, true, MODE_ROWS>(p, dev, st) : launch<128, false, MODE_ROWS>(p, dev, st);
        return bf16 ? launch<64, true, MODE_ROWS>(p, dev, st) : launch<64, false, MODE_ROWS>(p, dev, st);
    }
    if (raster) {
        if (D == 128)
            return bf16 ? launch<128, true, MODE_SQUARES>(p, dev, st) : launch<128, false, MODE_SQUARES>(p, dev, st);
        return bf16 ? launch<64, true, MODE_SQUARES>(p, dev, st) : launch<64, false, MODE_SQUARES>(p, dev, st);
    }
    if (D == 128) return bf16 ? launch<128, true, MODE_TILED>(p, dev, st) : launch<128, false, MODE_TILED>(p, dev, st);
    return bf16 ? launch<64, true, MODE_TILED>(p, dev, st) : launch<64, false, MODE_TILED>(p, dev, st);
}
}  // namespace
}  // namespace hb

extern "C" int hb_paired_fwd(const void* q, const void* k, const void* v, void* out, const int64_t* strides, int B,
                             int H, int N, int D, int G, int W, int key_block_size, const int32_t* kv_indices,
                             const int32_t* kv_flags, const int32_t* kv_counts, float scale_log2, int dtype,
                             const int32_t* row_map, void* workspace, size_t workspace_bytes, void* stream) {
    if (!out) return HB_ERR_ARG;
    return paired_fwd(q, k, v, out, strides, B, H, N, D, G, W, key_block_size, kv_indices, kv_flags, kv_counts,
                      scale_log2, dtype, row_map, nullptr, nullptr, workspace, workspace_bytes, stream);
}

extern "C" int hb_paired_fwd_raster(const void* q, const void* k, const void* v, void* out, const int64_t* strides,
                                    int B, int H, int N, int D, int G, int W, int key_block_size,
                                    const int32_t* kv_indices, const int32_t* kv_flags, const int32_t* kv_counts,
                                    float scale_log2, int dtype, const hb_raster_order_t* order, void* workspace,
                                    size_t workspace_bytes, void* stream) {
    if (!out || !order) return HB_ERR_ARG;
    return paired_fwd(q, k, v, out, strides, B, H, N, D, G, W, key_block_size, kv_indices, kv_flags, kv_counts,
                      scale_log2, dtype, nullptr, order, nullptr, workspace, workspace_bytes, stream);
}

extern "C" int hb_paired_fwd_allgather(const void* q, const void* k, const void* v, const int64_t* strides, int B,
                                       int H, int N, int D, int G, int W, int key_block_size,
                                       const int32_t* kv_indices, const int32_t* kv_flags, const int32_t* kv_counts,
                                       float scale_log2, int dtype, const hb_peer_out_t* peers, void* workspace,
                                       size_t workspace_bytes, void* stream) {
    if (!peers) return HB_ERR_ARG;
    return paired_fwd(q, k, v, nullptr, strides, B, H, N, D, G, W, key_block_size, kv_indices, kv_flags, kv_counts,
                      scale_log2, dtype, nullptr, nullptr, peers, workspace, workspace_bytes, stream);
}

// ---------------------------------------------------------------------------
// Allocation-free entry point.  For callers that cannot allocate device memory
// (runtime plugins that may not allocate while enqueueing, fixed-budget
// real-time hosts, bindings without a CUDA allocator): the scheduler words of
// the kernel live in this file-scope array instead of a caller workspace.
// Every GPU that loads the library holds its own copy until the process exits;
// all calls on a device share it, so overlapping calls race.
// ---------------------------------------------------------------------------
static __device__ __align__(256) int32_t hb_noalloc_scratch[HB_NOALLOC_SCRATCH_BYTES / 4];

namespace {
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {};

// Host code may not pass `hb_noalloc_scratch` itself to a kernel (on the host it
// names a stand-in, not device memory): look the device address up once per
// device, with that device current.
int noalloc_scratch(int dev, void** out) {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, hb_noalloc_scratch) != cudaSuccess || !p) return HB_ERR_CUDA;
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return HB_OK;
}
}  // namespace

extern "C" int hb_paired_fwd_noalloc(const void* q, const void* k, const void* v, void* out, const int64_t* strides,
                                     int B, int H, int N, int D, int G, int W, int key_block_size,
                                     const int32_t* kv_indices, const int32_t* kv_flags, const int32_t* kv_counts,
                                     float scale_log2, int dtype, void* stream) {
    if (B <= 0 || H <= 0 || N <= 0 || N % 128) return HB_ERR_ARG;
    if ((int64_t)B * H * (N / 128) > (int64_t)HB_NOALLOC_MAX_ITEMS) return HB_ERR_UNSUPPORTED;
    if (hb_fwd_workspace_bytes() > (size_t)HB_NOALLOC_SCRATCH_BYTES) return HB_ERR_WORKSPACE;
    int dev;
    HB_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return HB_ERR_UNSUPPORTED;
    void* scratch = nullptr;
    const int rc = noalloc_scratch(dev, &scratch);
    if (rc) return rc;
    // The work counter and finished-CTA counter must start at zero; the array
    // keeps whatever the previous call left, so clear it on the call's stream.
    HB_CUDA_TRY(cudaMemsetAsync(scratch, 0, hb_fwd_workspace_bytes(), (cudaStream_t)stream));
    // The array holds only the scheduler words, so long global rows run unsplit here.
    return hb_paired_fwd(q, k, v, out, strides, B, H, N, D, G, W, key_block_size, kv_indices, kv_flags, kv_counts,
                         scale_log2, dtype, nullptr, scratch, HB_NOALLOC_SCRATCH_BYTES, stream);
}
