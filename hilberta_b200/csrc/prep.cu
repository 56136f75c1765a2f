// Q/K/V preparation for the attention kernel: per-head RMSNorm, rotary embedding
// and the text + image concatenation in one pass over HBM.
//
// The FLUX processor (hilberta/flux_adapter.py:280-298) splits each projection
// into heads, RMS-normalises query and key rows over the head dimension with a
// learned weight (separate weights for the text and the image stream), puts the
// text tokens first, rotates query and key by the rotary embedding and hands
// [B, H, S, D] views of [B, S, H, D] storage to the attention.  As separate
// tensor ops that is four to five read+write passes per tensor; here every
// (token, head) row is read once and written once, straight into the [B, S, H, D]
// layout the attention kernel reads in place.
//
// Arithmetic follows those ops step by step (diffusers 0.36 RMSNorm and
// apply_rotary_emb with real cos/sin, the processor's dependency):
//   v   = mean over D of x^2 in fp32,     r = 1/sqrt(v + eps)
//   y   = round16(x * r)                  (the normalised row in the input dtype)
//   y   = round16(y * weight)             (weight in the input dtype)
//   out = round16(y[2i] * cos - y[2i+1] * sin),  round16(y[2i+1] * cos + y[2i] * sin)
// with each fp32 product and sum rounded separately (no fused multiply-add), as
// separate elementwise ops would (the sum of squares itself is accumulated in
// its own order).  Memory-bound: 16-byte accesses, four lanes per row, rows
// ordered head-fastest so one token's cos/sin serve all its heads from L1.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <climits>
#include <cstdint>

#include "common.cuh"

namespace hb {
namespace {

struct PrepParams {
    const void* txt;  // [B][T][H*D] (token stride txt_sn, batch stride txt_sb, elements)
    const void* img;  // [B][n][H*D]
    int64_t txt_sb, txt_sn, img_sb, img_sn;
    int B, T, n, H;
    const void* w_txt;  // [D] or null: no normalisation
    const void* w_img;
    float eps;
    const float* cos;  // [T + n][D] in output token order, or null: no rotation
    const float* sin;
    const int32_t* image_rows;  // [n] or null: image token i -> output token T + image_rows[i]
    void* out;                  // [B][S][H][D] with strides (o_sb, o_sn, o_sh)
    int64_t o_sb, o_sn, o_sh;
    int32_t* status;            // optional: bit HB_DEV_BAD_BLOCK for an out-of-range image row
};

// 16-bit pairs <-> fp32 (round to nearest even), two elements per instruction,
// and the product of two 16-bit pairs rounded once to 16 bits (the exact
// product of two 16-bit values fits in fp32, so this equals rounding the fp32
// product, as a 16-bit elementwise multiply does).
template <bool BF16>
struct Half16;
template <>
struct Half16<true> {
    static __device__ __forceinline__ void unpack(uint32_t u, float& a, float& b) {
        a = __uint_as_float(u << 16);
        b = __uint_as_float(u & 0xffff0000u);
    }
    static __device__ __forceinline__ uint32_t pack(float a, float b) {
        __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&v);
    }
    static __device__ __forceinline__ uint32_t mul(uint32_t a, uint32_t b) {
        __nv_bfloat162 r = __hmul2(*reinterpret_cast<__nv_bfloat162*>(&a), *reinterpret_cast<__nv_bfloat162*>(&b));
        return *reinterpret_cast<uint32_t*>(&r);
    }
};
template <>
struct Half16<false> {
    static __device__ __forceinline__ void unpack(uint32_t u, float& a, float& b) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u));
        a = f.x;
        b = f.y;
    }
    static __device__ __forceinline__ uint32_t pack(float a, float b) {
        __half2 v = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&v);
    }
    static __device__ __forceinline__ uint32_t mul(uint32_t a, uint32_t b) {
        __half2 r = __hmul2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
        return *reinterpret_cast<uint32_t*>(&r);
    }
};

// LPR lanes per (batch, token, head) row: lane l of the group owns the 16-byte
// chunks l, l+LPR, l+2*LPR, ... of the row, so each load instruction covers
// 16*LPR contiguous bytes of every row, while the row's sum of squares needs
// log2(LPR) shuffles and the 1/sqrt runs once per D/(8*LPR) chunks.  The row
// loop bound is the same for the whole block, so the shuffles always see a
// full warp.
template <int D, bool BF16, int LPR>
__global__ void __launch_bounds__(256) k_norm_rope_pack(const __grid_constant__ PrepParams p) {
    using H16 = Half16<BF16>;
    constexpr int CPL = D / (8 * LPR);  // 16-byte chunks per lane
    constexpr int RPB = 256 / LPR;      // rows per block iteration
    const int S = p.T + p.n;
    const int rows = p.B * S * p.H;
    const int half = threadIdx.x % LPR;  // lane within the row group
    const float inv_d = 1.f / D;  // a power of two: the product equals the division
    for (int row0 = blockIdx.x * RPB; row0 < rows; row0 += gridDim.x * RPB) {
        const int row = row0 + (threadIdx.x / LPR);
        const bool valid = row < rows;
        const int rr = valid ? row : 0;
        const int tok = rr / p.H;
        const int h = rr - tok * p.H;
        const int b = tok / S;
        const int s = tok - b * S;  // input token: text [0, T), then image
        const bool text = s < p.T;
        const uint16_t* src = (text ? static_cast<const uint16_t*>(p.txt) + (int64_t)b * p.txt_sb + (int64_t)s * p.txt_sn
                                    : static_cast<const uint16_t*>(p.img) + (int64_t)b * p.img_sb +
                                          (int64_t)(s - p.T) * p.img_sn) +
                              h * D + 8 * half;
        uint4 raw[CPL];
#pragma unroll
        for (int k = 0; k < CPL; k++)
            raw[k] = valid ? *reinterpret_cast<const uint4*>(src + 8 * LPR * k) : make_uint4(0, 0, 0, 0);
        float r = 1.f;
        const uint16_t* w = static_cast<const uint16_t*>(text ? p.w_txt : p.w_img);
        if (p.w_txt) {  // both weights or neither (checked on the host): uniform
            float ss = 0.f;
#pragma unroll
            for (int k = 0; k < CPL; k++) {
                const uint32_t u[4] = {raw[k].x, raw[k].y, raw[k].z, raw[k].w};
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    float a, c;
                    H16::unpack(u[i], a, c);
                    ss = fmaf(a, a, ss);
                    ss = fmaf(c, c, ss);
                }
            }
#pragma unroll
            for (int o = 1; o < LPR; o <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            r = 1.f / sqrtf(__fmul_rn(ss, inv_d) + p.eps);
        }
        if (!valid) continue;
        int so = s;  // output token
        if (!text && p.image_rows) {
            const int32_t m = p.image_rows[s - p.T];
            if (m < 0 || m >= p.n) {
                if (h == 0 && half == 0 && p.status) atomicOr(p.status, HB_DEV_BAD_BLOCK);
                continue;
            }
            so = p.T + m;
        }
        uint16_t* dst = static_cast<uint16_t*>(p.out) + (int64_t)b * p.o_sb + (int64_t)so * p.o_sn +
                        (int64_t)h * p.o_sh + 8 * half;
#pragma unroll
        for (int k = 0; k < CPL; k++) {
            const int col = 8 * LPR * k + 8 * half;  // first column of this chunk
            uint32_t u[4] = {raw[k].x, raw[k].y, raw[k].z, raw[k].w};
            if (p.w_txt) {
                const uint4 wr = *reinterpret_cast<const uint4*>(w + col);
                const uint32_t wu[4] = {wr.x, wr.y, wr.z, wr.w};
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    float a, c;
                    H16::unpack(u[i], a, c);
                    u[i] = H16::mul(H16::pack(__fmul_rn(a, r), __fmul_rn(c, r)), wu[i]);
                }
            }
            if (p.cos) {
                const float4* c4 = reinterpret_cast<const float4*>(p.cos + (int64_t)so * D + col);
                const float4* s4 = reinterpret_cast<const float4*>(p.sin + (int64_t)so * D + col);
                const float4 ca = c4[0], cb = c4[1], sa = s4[0], sb = s4[1];
                const float cs[8] = {ca.x, ca.y, ca.z, ca.w, cb.x, cb.y, cb.z, cb.w};
                const float sn[8] = {sa.x, sa.y, sa.z, sa.w, sb.x, sb.y, sb.z, sb.w};
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    float a, c;
                    H16::unpack(u[i], a, c);
                    u[i] = H16::pack(__fadd_rn(__fmul_rn(a, cs[2 * i]), __fmul_rn(-c, sn[2 * i])),
                                     __fadd_rn(__fmul_rn(c, cs[2 * i + 1]), __fmul_rn(a, sn[2 * i + 1])));
                }
            }
            *reinterpret_cast<uint4*>(dst + 8 * LPR * k) = make_uint4(u[0], u[1], u[2], u[3]);
        }
    }
}

}  // namespace
}  // namespace hb

using namespace hb;

extern "C" int hb_norm_rope_pack(const void* txt, int64_t txt_sb, int64_t txt_sn, const void* img, int64_t img_sb,
                                 int64_t img_sn, int B, int T, int n, int H, int D, const void* w_txt,
                                 const void* w_img, float eps, const float* cos, const float* sin,
                                 const int32_t* image_rows, void* out, int64_t o_sb, int64_t o_sn, int64_t o_sh,
                                 int dtype, int32_t* status, void* stream) {
    if (!out || B <= 0 || H <= 0 || T < 0 || n < 0 || T + n <= 0) return HB_ERR_ARG;
    if ((T > 0 && !txt) || (n > 0 && !img) || ((cos == nullptr) != (sin == nullptr))) return HB_ERR_ARG;
    if ((w_txt == nullptr) != (w_img == nullptr) || !(eps >= 0.f)) return HB_ERR_ARG;
    if (D != 64 && D != 128) return HB_ERR_UNSUPPORTED;
    if (dtype != 0 && dtype != 1) return HB_ERR_UNSUPPORTED;
    // 16-byte vector accesses: every row start and stride must keep them aligned
    auto a16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
    auto s8 = [](int64_t st) { return st % 8 == 0; };  // strides in 16-bit elements
    if ((txt && !a16(txt)) || (img && !a16(img)) || !a16(out) || (w_txt && (!a16(w_txt) || !a16(w_img))) ||
        (cos && (!a16(cos) || !a16(sin))) || (image_rows && (reinterpret_cast<uintptr_t>(image_rows) & 3)))
        return HB_ERR_ALIGN;
    if (!s8(txt_sb) || !s8(txt_sn) || !s8(img_sb) || !s8(img_sn) || !s8(o_sb) || !s8(o_sn) || !s8(o_sh))
        return HB_ERR_ALIGN;
    PrepParams p;
    p.txt = txt;
    p.img = img;
    p.txt_sb = txt_sb;
    p.txt_sn = txt_sn;
    p.img_sb = img_sb;
    p.img_sn = img_sn;
    p.B = B;
    p.T = T;
    p.n = n;
    p.H = H;
    p.w_txt = w_txt;
    p.w_img = w_img;
    p.eps = eps;
    p.cos = cos;
    p.sin = sin;
    p.image_rows = image_rows;
    p.out = out;
    p.o_sb = o_sb;
    p.o_sn = o_sn;
    p.o_sh = o_sh;
    p.status = status;
    int dev = 0, sms = 0;
    HB_CUDA_TRY(cudaGetDevice(&dev));
    HB_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int64_t rows = (int64_t)B * (T + n) * H;
    if (rows > INT32_MAX / 2) return HB_ERR_UNSUPPORTED;
    constexpr int LPR = 4;  // lanes per row (measured at 2048^2: 2 -> 0.168 ms, 4 -> 0.151, 8 -> 0.167 for Q+K+V)
    const int64_t want = (rows + 256 / LPR - 1) / (256 / LPR);
    const int grid = (int)(want < (int64_t)sms * 8 ? want : (int64_t)sms * 8);
    cudaStream_t st = (cudaStream_t)stream;
    if (D == 128) {
        if (dtype == 1)
            k_norm_rope_pack<128, true, LPR><<<grid, 256, 0, st>>>(p);
        else
            k_norm_rope_pack<128, false, LPR><<<grid, 256, 0, st>>>(p);
    } else {
        if (dtype == 1)
            k_norm_rope_pack<64, true, LPR><<<grid, 256, 0, st>>>(p);
        else
            k_norm_rope_pack<64, false, LPR><<<grid, 256, 0, st>>>(p);
    }
    HB_LAUNCH_CHECK();
    return HB_OK;
}
