// CUDA metadata builder: composite Hilbert order, shared-square packing, the four
// sliding tile phases, top-K cut-edge bridges (optionally closed reciprocally),
// per-row sorted K/V block lists, validation, paired (128-query) metadata and the
// dense correctness mask.  Integer-only; bit-exact with the reference builders:
//   hilberta/geometry.py:6-43, hilberta/plan.py:70-84 and :114-197,
//   hilberta/bridge_k.py:10-51, hilberta/sparse_kernel.py:100-166,
//   hilberta/paired_metadata.py:26-51.
#include <climits>
#include <cstdio>

#include "common.cuh"

namespace hb {
namespace {

constexpr unsigned FULL = 0xffffffffu;

// Raster id of the d-th cell of the grid's Hilbert walk, vertically flipped
// (geometry.py:6-25): per level s, rx = (t>>1)&1, ry = (t^rx)&1; a quadrant with
// ry == 0 is reflected when rx, then transposed; x += s*rx, y += s*ry.
__device__ inline int64_t hilbert_cell(int64_t d, int g) {
    int64_t x = 0, y = 0, t = d;
    for (int s = 1; s < g; s <<= 1) {
        const int64_t rx = (t >> 1) & 1;
        const int64_t ry = (t ^ rx) & 1;
        if (ry == 0) {
            if (rx) {
                x = s - 1 - x;
                y = s - 1 - y;
            }
            const int64_t tmp = x;
            x = y;
            y = tmp;
        }
        x += s * rx;
        y += s * ry;
        t >>= 2;
    }
    return (g - 1 - y) * (int64_t)g + x;
}

// Composite order (plan.py:133-135): the middle half of the Hilbert walk, then
// its point reflection n-1-h.  inv[original[i]] = i.
__global__ void k_composite(int g, int64_t n, int64_t* __restrict__ original, int32_t* __restrict__ inv) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int64_t half = n / 2, quarter = n / 4;
    const int64_t v = i < half ? hilbert_cell(quarter + i, g) : n - 1 - hilbert_cell(quarter + i - half, g);
    original[i] = v;
    inv[v] = (int32_t)i;
}

// Per original block: 0 = outside the shared square, 1 = inside, 2 = straddles
// (plan.py:138-145; the square is rows/cols [3g/8, 5g/8) of the raster grid).
__global__ void k_share_flags(int g, int b, int64_t nb, int shared, const int64_t* __restrict__ original,
                              int32_t* __restrict__ share, int32_t* __restrict__ info) {
    const int64_t kb = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (kb >= nb) return;
    int cnt = 0;
    if (shared) {
        const int s0 = 3 * g / 8, s1 = 5 * g / 8;
        for (int i = 0; i < b; i++) {
            const int64_t a = original[kb * b + i];
            const int y = (int)(a / g), x = (int)(a % g);
            cnt += (y >= s0 && y < s1 && x >= s0 && x < s1);
        }
    }
    share[kb] = cnt == 0 ? 0 : (cnt == b ? 1 : 2);
    if (cnt != 0 && cnt != b) atomicCAS(&info[0], 0, HB_ERR_SHARED);
}

// Block-wide exclusive scan of one int per thread (blockDim.x multiple of 32, <= 1024).
__device__ int block_exclusive_scan(int v, int* warp_sums, int* total) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(FULL, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[w] = x;
    __syncthreads();
    if (w == 0) {
        int s = lane < nw ? warp_sums[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(FULL, s, o);
            if (lane >= o) s += y;
        }
        warp_sums[lane] = s;
    }
    __syncthreads();
    const int excl = x - v + (w > 0 ? warp_sums[w - 1] : 0);
    *total = warp_sums[nw - 1];
    __syncthreads();
    return excl;
}

// Physical block order = shared blocks then ordinary blocks, each ascending by
// original id (plan.py:145-150).  packed[p] = original id; o2p[kb] = physical
// block id (text blocks first).  One CTA of 1024 threads.  Straddling blocks
// (an error the host reports from info[0]) are packed with the ordinary ones so
// that packed / o2p stay permutations and no later kernel indexes out of range.
__global__ void k_pack(int64_t nb, int64_t text_blocks, const int32_t* __restrict__ share,
                       int64_t* __restrict__ packed, int32_t* __restrict__ o2p, int32_t* __restrict__ info) {
    __shared__ int warp_sums[32];
    int base = 0;
    for (int pass = 0; pass < 2; pass++) {
        for (int64_t c = 0; c < nb; c += blockDim.x) {
            const int64_t kb = c + threadIdx.x;
            const int f = (kb < nb && ((share[kb] == 1) == (pass == 0))) ? 1 : 0;
            int total;
            const int pos = base + block_exclusive_scan(f, warp_sums, &total);
            if (f) {
                packed[pos] = kb;
                o2p[kb] = (int32_t)(pos + text_blocks);
            }
            base += total;
        }
        if (pass == 0 && threadIdx.x == 0) info[1] = base;
    }
}

// Token order of the persistent layout: blocks in physical order (plan.py:147).
__global__ void k_image_order(int b, int64_t n, const int64_t* __restrict__ original, const int64_t* __restrict__ packed,
                              int64_t* __restrict__ order, int64_t* __restrict__ inv_order) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int64_t v = original[packed[i / b] * b + i % b];
    order[i] = v;
    inv_order[v] = i;
}

__device__ inline int64_t tile_label(int64_t pos, int64_t off, int64_t n, int64_t width) {
    return pymod(pos - off, n) / width;
}

// One warp per (original query block q, phase): score every other block by the
// number of 4-neighbour pixel pairs between them that the phase's tiling cuts
// (plan.py:160-166, bridge_k.py:22-28), then pick the top K by
// (-score, (key - offset/b) mod nb) (plan.py:167-172, bridge_k.py:36-43).
// Also asserts that no block straddles a tile boundary (plan.py:156-158).
__global__ void k_bridge(int g, int b, int64_t n, int64_t nb, int64_t width, int K, const int64_t* __restrict__ original,
                         const int32_t* __restrict__ inv, int32_t* __restrict__ chosen, int64_t* __restrict__ chosen_out,
                         int32_t* __restrict__ info) {
    extern __shared__ int cand[];  // up to 4*b candidate block ids
    __shared__ int m;
    __shared__ int picks[4];
    const int lane = threadIdx.x;
    const int64_t q = blockIdx.x;
    const int ph = blockIdx.y;
    const int64_t off = ph * (width / 4);
    const int64_t offb = off / b;
    if (lane == 0) m = 0;
    __syncwarp();
    const int64_t lq = tile_label(q * b, off, n, width);
    for (int i = lane; i < b; i += 32) {
        if (tile_label(q * b + i, off, n, width) != lq) atomicCAS(&info[0], 0, HB_ERR_CROSS);
        const int64_t a = original[q * b + i];
        const int y = (int)(a / g), x = (int)(a % g);
        for (int dir = 0; dir < 4; dir++) {
            int64_t r;
            if (dir == 0) {
                if (x == 0) continue;
                r = a - 1;
            } else if (dir == 1) {
                if (x + 1 >= g) continue;
                r = a + 1;
            } else if (dir == 2) {
                if (y == 0) continue;
                r = a - g;
            } else {
                if (y + 1 >= g) continue;
                r = a + g;
            }
            const int64_t pr = inv[r];
            if (tile_label(pr, off, n, width) != lq) cand[atomicAdd(&m, 1)] = (int)(pr / b);
        }
    }
    __syncwarp();
    const int mm = m;
    for (int r = 0; r < K; r++) {
        unsigned long long best = 0ull;
        for (int i = lane; i < mm; i += 32) {
            const int c = cand[i];
            int score = 0;
            bool first = true;
            for (int j = 0; j < mm; j++) {
                if (cand[j] == c) {
                    score++;
                    if (j < i) first = false;
                }
            }
            bool taken = false;
            for (int t = 0; t < r; t++) taken |= picks[t] == c;
            if (!first || taken) continue;
            const uint32_t tie = (uint32_t)pymod(c - offb, nb);
            const unsigned long long key = ((unsigned long long)score << 32) | (unsigned long long)(0xffffffffu - tie);
            best = best > key ? best : key;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(FULL, best, o);
            best = best > other ? best : other;
        }
        if (lane == 0) {
            int sel = -1;
            if (best != 0ull) {
                const uint32_t tie = 0xffffffffu - (uint32_t)(best & 0xffffffffull);
                sel = (int)pymod((int64_t)tie + offb, nb);
            }
            picks[r] = sel;
        }
        __syncwarp();
    }
    if (lane < K) {
        const int64_t o = ((int64_t)ph * nb + q) * K + lane;
        chosen[o] = picks[lane];
        chosen_out[o] = picks[lane];
    }
}

__global__ void k_hilbert(int g, int64_t n, int64_t* __restrict__ out) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i < n) out[i] = hilbert_cell(i, g);
}

__global__ void k_fill_i64(int64_t* p, int64_t count, int64_t v) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i < count) p[i] = v;
}

// Write the ascending ids of the set bytes of bits[0..total) into out[0..cap),
// zero padded; returns the count (valid in thread 0).
__device__ int compact_bytes(const unsigned char* bits, int64_t total, int32_t* out, int64_t cap, const int32_t* flags_in,
                             int32_t* flags_out) {
    __shared__ int warp_sums[32];
    const int64_t chunk = ceil_div(total, blockDim.x);
    const int64_t s = threadIdx.x * chunk;
    const int64_t e = s + chunk < total ? s + chunk : total;
    int local = 0;
    for (int64_t i = s; i < e; i++) local += bits[i] != 0;
    int count;
    int pos = block_exclusive_scan(local, warp_sums, &count);
    for (int64_t i = s; i < e; i++) {
        if (bits[i]) {
            out[pos] = (int32_t)i;
            if (flags_out) flags_out[pos] = flags_in[i];
            pos++;
        }
    }
    for (int64_t i = count + threadIdx.x; i < cap; i += blockDim.x) {
        out[i] = 0;
        if (flags_out) flags_out[i] = 0;
    }
    return count;
}

// One CTA per (ordinary row, phase): global blocks, same-tile ordinary blocks
// (plan.py:173-184), the row's own bridges and, when reciprocal, every block
// that chose this one (bridge_k.py:44 adj | adj.T), emitted ascending
// (bridge_k.py:45-49).
__global__ void k_rows(int b, int64_t n, int64_t nb, int64_t width, int64_t text_blocks, int64_t n_share, int64_t rows,
                       int64_t total, int64_t cap, int K, int reciprocal, const int32_t* __restrict__ share,
                       const int64_t* __restrict__ packed, const int32_t* __restrict__ o2p,
                       const int32_t* __restrict__ chosen, int32_t* __restrict__ kv, int32_t* __restrict__ counts,
                       int32_t* __restrict__ info) {
    extern __shared__ unsigned char bits[];
    const int64_t row = blockIdx.x;
    const int ph = blockIdx.y;
    const int64_t off = ph * (width / 4);
    const int64_t gb = text_blocks + n_share;
    const int64_t q = packed[n_share + row];
    for (int64_t i = threadIdx.x; i < total; i += blockDim.x) bits[i] = i < gb;
    __syncthreads();
    const int64_t lq = tile_label(q * b, off, n, width);
    for (int64_t kb = threadIdx.x; kb < nb; kb += blockDim.x)
        if (share[kb] == 0 && tile_label(kb * b, off, n, width) == lq) bits[o2p[kb]] = 1;
    if (K > 0) {
        const int32_t* ch = chosen + (int64_t)ph * nb * K;
        if (threadIdx.x < K) {
            const int c = ch[q * K + threadIdx.x];
            if (c >= 0) bits[o2p[c]] = 1;
        }
        if (reciprocal)
            for (int64_t qq = threadIdx.x; qq < nb; qq += blockDim.x)
                for (int j = 0; j < K; j++)
                    if (ch[qq * K + j] == q) bits[o2p[qq]] = 1;
    }
    __syncthreads();
    int32_t* out = kv + ((int64_t)ph * rows + row) * cap;
    const int count = compact_bytes(bits, total, out, cap, nullptr, nullptr);
    if (threadIdx.x == 0) {
        counts[(int64_t)ph * rows + row] = count;
        atomicMax(&info[2 + ph], count);
    }
}

__global__ void k_validate_init(int32_t* res) {
    res[0] = INT_MAX;
    res[1] = INT_MAX;
    res[2] = INT_MIN;
    res[3] = 0;
}

// validate_metadata (sparse_kernel.py:136-145) for one row per CTA.
__global__ void k_validate(const int32_t* __restrict__ ids, int64_t ld, int width, const int32_t* __restrict__ counts,
                           int nblocks, int gblocks, int32_t* __restrict__ res) {
    extern __shared__ uint32_t seen[];
    __shared__ int bad_range, bad_glob;
    const int row = blockIdx.x;
    const int words = (nblocks + 31) / 32;
    for (int i = threadIdx.x; i < words; i += blockDim.x) seen[i] = 0;
    if (threadIdx.x == 0) bad_range = bad_glob = 0;
    __syncthreads();
    const int c = counts[row];
    if (c < 1 || c > width) {
        if (threadIdx.x == 0) atomicMin(&res[0], row * 4 + 1);
        return;
    }
    for (int i = threadIdx.x; i < c; i += blockDim.x) {
        const int v = ids[(int64_t)row * ld + i];
        if (v < 0 || v >= nblocks) {
            bad_range = 1;
        } else {
            const uint32_t bit = 1u << (v & 31);
            if (atomicOr(&seen[v >> 5], bit) & bit) bad_range = 1;
        }
    }
    __syncthreads();
    if (bad_range) {
        if (threadIdx.x == 0) atomicMin(&res[0], row * 4 + 2);
        return;
    }
    for (int i = threadIdx.x; i < gblocks; i += blockDim.x)
        if (!(seen[i >> 5] & (1u << (i & 31)))) bad_glob = 1;
    __syncthreads();
    if (threadIdx.x == 0) {
        if (bad_glob) atomicMin(&res[0], row * 4 + 3);
        atomicMin(&res[1], c);
        atomicMax(&res[2], c);
        atomicAdd(&res[3], c);
    }
}

// pair_metadata (paired_metadata.py:26-51): union of rows 2i, 2i+1; flag bit
// (half + 2*key_half) per contributing 64-token query half / key half.
__global__ void k_pair(const int32_t* __restrict__ ids, int64_t ld, const int32_t* __restrict__ counts, int ratio,
                       int64_t nkb, int32_t* __restrict__ out_ids, int32_t* __restrict__ out_flags, int64_t ld_out,
                       int32_t* __restrict__ out_counts, int32_t* __restrict__ info) {
    extern __shared__ int32_t fl[];
    unsigned char* bits = reinterpret_cast<unsigned char*>(fl + nkb);
    const int64_t pr = blockIdx.x;
    for (int64_t i = threadIdx.x; i < nkb; i += blockDim.x) fl[i] = 0;
    __syncthreads();
    for (int half = 0; half < 2; half++) {
        const int64_t r = 2 * pr + half;
        const int c = counts[r];
        for (int i = threadIdx.x; i < c; i += blockDim.x) {
            const int blk = ids[r * ld + i];
            if (blk >= 0 && blk / ratio < nkb) atomicOr(&fl[blk / ratio], 1 << (half + 2 * (blk % ratio)));
        }
    }
    __syncthreads();
    for (int64_t i = threadIdx.x; i < nkb; i += blockDim.x) bits[i] = fl[i] != 0;
    __syncthreads();
    const int count = compact_bytes(bits, nkb, out_ids + pr * ld_out, ld_out, fl, out_flags + pr * ld_out);
    if (threadIdx.x == 0) {
        out_counts[pr] = count;
        atomicMax(&info[0], count);
    }
}

// KV128 paired rows -> the equivalent KV64 rows.  A KV128 entry (block b, flag
// bits half + 2*key_half, paired_metadata.py:26-51) covers 64-key blocks 2b and
// 2b+1; each half with any query-half bit becomes one KV64 entry whose bits 0/1
// are that half's.  One warp per paired row; entries stay ascending, so the
// result is the row pair_metadata builds for key_block_size 64.  Counts are
// clamped to [0, width]; flag bits above 3 are ignored.
__global__ void k_expand_kv128(const int32_t* __restrict__ ids, const int32_t* __restrict__ flags, int64_t ld,
                               int width, const int32_t* __restrict__ counts, int rows, int32_t* __restrict__ out_ids,
                               int32_t* __restrict__ out_flags, int64_t ld_out, int32_t* __restrict__ out_counts) {
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const int c = min(max(counts[row], 0), width);
    int base = 0;
    for (int e0 = 0; e0 < c; e0 += 32) {
        const int e = e0 + lane;
        int blk = 0, f = 0;
        if (e < c) {
            blk = ids[row * ld + e];
            f = flags[row * ld + e] & 15;
        }
        const int lo = f & 3, hi = (f >> 2) & 3;
        const int n = (lo != 0) + (hi != 0);
        int incl = n;  // inclusive warp scan of the entries each lane emits
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t;
        }
        int pos = base + incl - n;
        if (lo) {
            out_ids[row * ld_out + pos] = 2 * blk;
            out_flags[row * ld_out + pos] = lo;
            pos++;
        }
        if (hi) {
            out_ids[row * ld_out + pos] = 2 * blk + 1;
            out_flags[row * ld_out + pos] = hi;
        }
        base += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) out_counts[row] = base;
}

// Dense token mask, one CTA per 64-row (block_size) query block (plan.py:70-84).
__global__ void k_dense_mask(const int32_t* __restrict__ ids, int64_t ld, const int32_t* __restrict__ counts, int tokens,
                             int global_tokens, int bs, uint8_t* __restrict__ mask) {
    extern __shared__ unsigned char allowed[];  // tokens / bs
    const int rb = blockIdx.x;
    const int nbc = tokens / bs;
    const int gbr = global_tokens / bs;
    for (int i = threadIdx.x; i < nbc; i += blockDim.x) allowed[i] = rb < gbr;
    __syncthreads();
    if (rb >= gbr) {
        const int r = rb - gbr;
        const int c = counts[r];
        for (int i = threadIdx.x; i < c; i += blockDim.x) {
            const int id = ids[(int64_t)r * ld + i];
            if (id >= 0 && id < nbc) allowed[id] = 1;
        }
    }
    __syncthreads();
    for (int rr = 0; rr < bs; rr++) {
        uint8_t* dst = mask + ((int64_t)rb * bs + rr) * tokens;
        for (int col = threadIdx.x; col < tokens; col += blockDim.x) dst[col] = allowed[col / bs];
    }
}

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

}  // namespace
}  // namespace hb

using namespace hb;

extern "C" int hb_hilbert_order(int grid_size, int64_t* out, void* stream_) {
    if (!out || grid_size < 2 || !is_pow2(grid_size) || grid_size > 65536) return HB_ERR_ARG;
    const int64_t n = (int64_t)grid_size * grid_size;
    k_hilbert<<<(unsigned)ceil_div(n, 256), 256, 0, (cudaStream_t)stream_>>>(grid_size, n, out);
    HB_LAUNCH_CHECK();
    return HB_OK;
}

extern "C" int hb_plan_dims(int grid_size, int tile_count, int text_tokens, int block_size, int shared,
                            hb_plan_dims_t* out) {
    if (!out) return HB_ERR_ARG;
    if (grid_size <= 0 || tile_count <= 0 || text_tokens <= 0 || block_size <= 0) return HB_ERR_ARG;
    if (grid_size < 8 || !is_pow2(grid_size) || grid_size > 4096) return HB_ERR_ARG;
    const int64_t g = grid_size, n = g * g;
    if (n % tile_count || (n / tile_count) % (4 * (int64_t)block_size) || text_tokens % block_size) return HB_ERR_ALIGN;
    const int64_t nb = n / block_size;
    int64_t nshare = 0;
    if (shared) {
        const int64_t side = 5 * g / 8 - 3 * g / 8;
        if ((side * side) % block_size) return HB_ERR_SHARED;
        nshare = side * side / block_size;
    }
    out->image_tokens = n;
    out->image_blocks = nb;
    out->text_blocks = text_tokens / block_size;
    out->total_blocks = out->text_blocks + nb;
    out->shared_blocks = nshare;
    out->rows = nb - nshare;
    out->row_capacity = out->total_blocks;
    out->workspace_bytes =
        (int64_t)(align256(4 * (size_t)n) + 2 * align256(4 * (size_t)nb) + align256(4 * 4 * (size_t)nb * 4));
    return HB_OK;
}

extern "C" int hb_plan_build(int grid_size, int tile_count, int text_tokens, int block_size, int shared, int bridge_k,
                             int reciprocal, int64_t* image_order, int64_t* inverse_image_order,
                             int64_t* original_order, int64_t* physical_original_blocks, int32_t* kv_indices,
                             int32_t* kv_counts, int64_t* bridge_original_blocks, int32_t* info, void* workspace,
                             size_t workspace_bytes, void* stream_) {
    hb_plan_dims_t d;
    const int rc = hb_plan_dims(grid_size, tile_count, text_tokens, block_size, shared, &d);
    if (rc) return rc;
    if (bridge_k < 0 || bridge_k > 4 || (reciprocal != 0 && reciprocal != 1) || (!reciprocal && bridge_k > 1))
        return HB_ERR_ARG;
    if (!image_order || !inverse_image_order || !original_order || !physical_original_blocks || !kv_indices ||
        !kv_counts || !bridge_original_blocks || !info || !workspace)
        return HB_ERR_ARG;
    if (workspace_bytes < (size_t)d.workspace_bytes) return HB_ERR_WORKSPACE;
    if (4 * (int64_t)block_size * 4 > 48 * 1024 || d.total_blocks > 48 * 1024) return HB_ERR_UNSUPPORTED;
    cudaStream_t st = (cudaStream_t)stream_;
    const int64_t n = d.image_tokens, nb = d.image_blocks, width = n / tile_count;
    char* ws = (char*)workspace;
    int32_t* inv = (int32_t*)ws;
    ws += align256(4 * (size_t)n);
    int32_t* share = (int32_t*)ws;
    ws += align256(4 * (size_t)nb);
    int32_t* o2p = (int32_t*)ws;
    ws += align256(4 * (size_t)nb);
    int32_t* chosen = (int32_t*)ws;
    const int K = bridge_k;
    const int kout = K > 0 ? K : 1;

    HB_CUDA_TRY(cudaMemsetAsync(info, 0, 8 * sizeof(int32_t), st));
    const int T = 256;
    k_composite<<<(unsigned)ceil_div(n, T), T, 0, st>>>(grid_size, n, original_order, inv);
    k_share_flags<<<(unsigned)ceil_div(nb, T), T, 0, st>>>(grid_size, block_size, nb, shared, original_order, share, info);
    k_pack<<<1, 1024, 0, st>>>(nb, d.text_blocks, share, physical_original_blocks, o2p, info);
    k_image_order<<<(unsigned)ceil_div(n, T), T, 0, st>>>(block_size, n, original_order, physical_original_blocks,
                                                            image_order, inverse_image_order);
    if (K > 0) {
        k_bridge<<<dim3((unsigned)nb, 4), 32, 4 * block_size * sizeof(int), st>>>(
            grid_size, block_size, n, nb, width, K, original_order, inv, chosen, bridge_original_blocks, info);
    } else {
        k_fill_i64<<<(unsigned)ceil_div(4 * nb, T), T, 0, st>>>(bridge_original_blocks, 4 * nb, -1);
    }
    HB_LAUNCH_CHECK();
    k_rows<<<dim3((unsigned)d.rows, 4), T, (size_t)d.total_blocks, st>>>(
        block_size, n, nb, width, d.text_blocks, d.shared_blocks, d.rows, d.total_blocks, d.row_capacity, K,
        reciprocal, share, physical_original_blocks, o2p, chosen, kv_indices, kv_counts, info);
    (void)kout;
    HB_LAUNCH_CHECK();
    return HB_OK;
}

extern "C" int hb_validate_metadata(const int32_t* kv_indices, int64_t ld, int32_t width, const int32_t* kv_counts,
                                    int32_t rows, int32_t tokens, int32_t global_tokens, int32_t* result,
                                    void* stream_) {
    if (!kv_indices || !kv_counts || !result || rows <= 0 || width < 1 || ld < width) return HB_ERR_ARG;
    if (tokens <= 0 || tokens % 64 || global_tokens < 0 || global_tokens % 64 || global_tokens >= tokens)
        return HB_ERR_ARG;
    cudaStream_t st = (cudaStream_t)stream_;
    const int nblocks = tokens / 64;
    k_validate_init<<<1, 1, 0, st>>>(result);
    k_validate<<<rows, 128, ((nblocks + 31) / 32) * sizeof(uint32_t), st>>>(kv_indices, ld, width, kv_counts, nblocks,
                                                                              global_tokens / 64, result);
    HB_LAUNCH_CHECK();
    return HB_OK;
}

extern "C" int hb_pair_metadata(const int32_t* kv_indices, int64_t ld, const int32_t* kv_counts, int32_t rows,
                                int32_t tokens, int32_t global_tokens, int32_t key_block_size, int32_t* out_ids,
                                int32_t* out_flags, int64_t ld_out, int32_t* out_counts, int32_t* info,
                                void* stream_) {
    if (!kv_indices || !kv_counts || !out_ids || !out_flags || !out_counts || !info) return HB_ERR_ARG;
    if ((key_block_size != 64 && key_block_size != 128) || tokens % 128 || global_tokens % 128 || rows <= 0 ||
        rows % 2)
        return HB_ERR_ARG;
    const int ratio = key_block_size / 64;
    const int64_t nkb = ceil_div(tokens / 64, ratio);
    if (ld_out < nkb) return HB_ERR_ARG;
    const size_t smem = (size_t)nkb * 5;
    if (smem > 200 * 1024) return HB_ERR_UNSUPPORTED;
    cudaStream_t st = (cudaStream_t)stream_;
    if (smem > 48 * 1024)
        HB_CUDA_TRY(cudaFuncSetAttribute(k_pair, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    HB_CUDA_TRY(cudaMemsetAsync(info, 0, sizeof(int32_t), st));
    k_pair<<<rows / 2, 256, smem, st>>>(kv_indices, ld, kv_counts, ratio, nkb, out_ids, out_flags, ld_out, out_counts,
                                        info);
    HB_LAUNCH_CHECK();
    return HB_OK;
}

extern "C" int hb_expand_kv128(const int32_t* kv_indices, const int32_t* kv_flags, int64_t ld, int32_t width,
                               const int32_t* kv_counts, int32_t rows, int32_t* out_ids, int32_t* out_flags,
                               int64_t ld_out, int32_t* out_counts, void* stream_) {
    if (rows < 0 || width < 1 || ld < width || ld_out < 2 * (int64_t)width) return HB_ERR_ARG;
    if (rows == 0) return HB_OK;
    if (!kv_indices || !kv_flags || !kv_counts || !out_ids || !out_flags || !out_counts) return HB_ERR_ARG;
    constexpr int kWarps = 8;
    k_expand_kv128<<<(rows + kWarps - 1) / kWarps, 32 * kWarps, 0, (cudaStream_t)stream_>>>(
        kv_indices, kv_flags, ld, width, kv_counts, rows, out_ids, out_flags, ld_out, out_counts);
    HB_LAUNCH_CHECK();
    return HB_OK;
}

extern "C" int hb_dense_mask(const int32_t* kv_indices, int64_t ld, const int32_t* kv_counts, int32_t rows,
                             int32_t tokens, int32_t global_tokens, int32_t block_size, uint8_t* mask, void* stream_) {
    if (!mask || block_size <= 0 || tokens % block_size || global_tokens % block_size ||
        rows != (tokens - global_tokens) / block_size)
        return HB_ERR_ARG;
    if (rows > 0 && (!kv_indices || !kv_counts)) return HB_ERR_ARG;
    const int nbc = tokens / block_size;
    if (nbc > 48 * 1024) return HB_ERR_UNSUPPORTED;
    k_dense_mask<<<nbc, 256, (size_t)nbc, (cudaStream_t)stream_>>>(kv_indices, ld, kv_counts, tokens, global_tokens,
                                                                    block_size, mask);
    HB_LAUNCH_CHECK();
    return HB_OK;
}

extern "C" const char* hb_status_string(int code) {
    switch (code) {
        case HB_OK: return "ok";
        case HB_ERR_ARG: return "invalid argument";
        case HB_ERR_ALIGN: return "Tile quarter offsets and text prefix must be block aligned";
        case HB_ERR_SHARED: return "Shared square must be a union of complete original blocks";
        case HB_ERR_CROSS: return "A physical block crosses a tile boundary";
        case HB_ERR_CUDA: return "CUDA runtime error";
        case HB_ERR_WORKSPACE: return "workspace too small";
        case HB_ERR_UNSUPPORTED: return "shape or dtype outside the compiled kernels";
        case HB_ERR_DEVICE: return "kernel reported a device status";
        case HB_ERR_TMA: return "TMA tensor map rejected the tensor (16-byte aligned base and strides required)";
        default: return "unknown status";
    }
}

extern "C" int hb_version(void) { return 100; }
