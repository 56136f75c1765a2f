// Adaptive-LayerNorm modulation and gated residuals of the FLUX transformer
// blocks around the attention (the adaLN-Zero steps of diffusers'
// FluxTransformerBlock / FluxSingleTransformerBlock, which wrap the processor of
// hilberta/flux_adapter.py:259-340):
//
//   x' = x + gate[b] * y                         (gated residual, optional)
//   h  = LayerNorm(x') * (1 + scale[b]) + shift[b]   (LayerNorm without affine, optional)
//
// As tensor ops these are five to seven read+write passes over the [tokens,
// hidden] stream (the LayerNorm, the broadcast multiply and add of the
// modulation, the gate multiply and the residual add).  Here one warp owns one
// row: the row is read once (plus y when the residual is taken), kept in
// registers, and x' and h are each written once.
//
// Arithmetic: fp32 throughout; x' is rounded to the 16-bit type before the
// LayerNorm reads it (it is the stored residual stream); mean and variance by
// two passes over the register-held row, 1/sqrt(var + eps) by rsqrtf, and h
// rounded once.  Memory-bound: 16-byte accesses, C a multiple of 256 (8
// elements per lane per vector) up to 4096.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "common.cuh"

namespace hb {
namespace {

constexpr int kMaxVec = 16;  // vectors of 8 elements per lane: C <= 32 * 8 * 16 = 4096

struct AdaParams {
    const void* x;  // [rows][C], row stride x_rs (elements)
    const void* y;  // [rows][C] or null, row stride y_rs
    const void* gate;   // [B][C] (batch stride mod_bs) when y is given
    const void* shift;  // [B][C] when h is written
    const void* scale;
    void* x_out;  // [rows][C] (may alias x) when y is given
    void* h_out;  // [rows][C] or null
    int64_t x_rs, y_rs, xo_rs, h_rs, mod_bs;
    int rows, rows_per_batch, C;
    float eps;
};

template <bool BF16>
struct Vec8 {
    using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
    static __device__ __forceinline__ void load(const void* p, float (&f)[8]) {
        const uint4 u = *reinterpret_cast<const uint4*>(p);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if constexpr (BF16) {
                f[2 * i] = __uint_as_float(w[i] << 16);
                f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
            } else {
                const __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
                const float2 t = __half22float2(h);
                f[2 * i] = t.x;
                f[2 * i + 1] = t.y;
            }
        }
    }
    static __device__ __forceinline__ uint4 pack(const float (&f)[8]) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if constexpr (BF16) {
                const __nv_bfloat162 b = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
                w[i] = *reinterpret_cast<const uint32_t*>(&b);
            } else {
                const __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
                w[i] = *reinterpret_cast<const uint32_t*>(&h);
            }
        }
        return make_uint4(w[0], w[1], w[2], w[3]);
    }
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// One warp per row; lane l owns elements [8 (l + 32 i), 8 (l + 32 i) + 8) for
// i < C / 256, so each 16-byte vector access of a warp covers 512 contiguous bytes.
template <bool BF16, bool RESIDUAL, bool NORM>
__global__ void __launch_bounds__(256) k_adaln(AdaParams p) {
    using V = Vec8<BF16>;
    using T = typename V::T;
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (row >= p.rows) return;  // whole warps leave together
    const int b = row / p.rows_per_batch;
    const int nv = p.C >> 8;
    const T* x = static_cast<const T*>(p.x) + row * p.x_rs;
    uint4 xv[kMaxVec];
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i)
        if (i < nv) xv[i] = *reinterpret_cast<const uint4*>(x + 8 * (lane + 32 * i));
    if constexpr (RESIDUAL) {
        const T* y = static_cast<const T*>(p.y) + row * p.y_rs;
        const T* g = static_cast<const T*>(p.gate) + b * p.mod_bs;
        T* xo = static_cast<T*>(p.x_out) + row * p.xo_rs;
#pragma unroll
        for (int i = 0; i < kMaxVec; ++i) {
            if (i < nv) {
                const int c = 8 * (lane + 32 * i);
                float fx[8], fy[8], fg[8];
                V::load(&xv[i], fx);
                V::load(y + c, fy);
                V::load(g + c, fg);
#pragma unroll
                for (int e = 0; e < 8; ++e) fx[e] = fmaf(fg[e], fy[e], fx[e]);
                xv[i] = V::pack(fx);  // the stored residual stream, rounded
                *reinterpret_cast<uint4*>(xo + c) = xv[i];
            }
        }
    }
    if constexpr (NORM) {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < kMaxVec; ++i) {
            if (i < nv) {
                float f[8];
                V::load(&xv[i], f);
#pragma unroll
                for (int e = 0; e < 8; ++e) s += f[e];
            }
        }
        const float inv_c = 1.f / static_cast<float>(p.C);
        const float mean = warp_sum(s) * inv_c;
        float q = 0.f;
#pragma unroll
        for (int i = 0; i < kMaxVec; ++i) {
            if (i < nv) {
                float f[8];
                V::load(&xv[i], f);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const float d = f[e] - mean;
                    q = fmaf(d, d, q);
                }
            }
        }
        const float rstd = rsqrtf(warp_sum(q) * inv_c + p.eps);
        const T* sh = static_cast<const T*>(p.shift) + b * p.mod_bs;
        const T* sc = static_cast<const T*>(p.scale) + b * p.mod_bs;
        T* h = static_cast<T*>(p.h_out) + row * p.h_rs;
#pragma unroll
        for (int i = 0; i < kMaxVec; ++i) {
            if (i < nv) {
                const int c = 8 * (lane + 32 * i);
                float f[8], fs[8], fc[8];
                V::load(&xv[i], f);
                V::load(sh + c, fs);
                V::load(sc + c, fc);
#pragma unroll
                for (int e = 0; e < 8; ++e) f[e] = fmaf((f[e] - mean) * rstd, 1.f + fc[e], fs[e]);
                *reinterpret_cast<uint4*>(h + c) = V::pack(f);
            }
        }
    }
}

template <bool BF16>
int launch_adaln(const AdaParams& p, cudaStream_t st) {
    const dim3 grid((p.rows + 7) / 8), block(256);
    const bool res = p.y != nullptr, norm = p.h_out != nullptr;
    if (res && norm)
        k_adaln<BF16, true, true><<<grid, block, 0, st>>>(p);
    else if (res)
        k_adaln<BF16, true, false><<<grid, block, 0, st>>>(p);
    else
        k_adaln<BF16, false, true><<<grid, block, 0, st>>>(p);
    HB_CUDA_TRY(cudaGetLastError());
    return HB_OK;
}

}  // namespace
}  // namespace hb

extern "C" int hb_adaln_residual(const void* x, int64_t x_rs, const void* y, int64_t y_rs, const void* gate,
                                 const void* shift, const void* scale, int64_t mod_bs, void* x_out, int64_t xo_rs,
                                 void* h_out, int64_t h_rs, int rows, int rows_per_batch, int C, float eps, int dtype,
                                 void* stream) {
    using namespace hb;
    if (!x || rows < 0 || rows_per_batch <= 0 || C <= 0 || !(eps >= 0.f)) return HB_ERR_ARG;
    if (!y && !h_out) return HB_ERR_ARG;                 // nothing to do
    if (y && (!gate || !x_out)) return HB_ERR_ARG;       // residual needs its gate and destination
    if (h_out && (!shift || !scale)) return HB_ERR_ARG;  // modulation needs shift and scale
    if (dtype != 0 && dtype != 1) return HB_ERR_UNSUPPORTED;
    if (C % 256 || C > 256 * kMaxVec) return HB_ERR_UNSUPPORTED;
    auto a16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
    auto s8 = [](int64_t st) { return st % 8 == 0; };
    if (!a16(x) || (y && (!a16(y) || !a16(gate) || !a16(x_out))) || (h_out && (!a16(h_out) || !a16(shift) || !a16(scale))))
        return HB_ERR_ALIGN;
    if (!s8(x_rs) || !s8(y_rs) || !s8(xo_rs) || !s8(h_rs) || !s8(mod_bs)) return HB_ERR_ALIGN;
    if (rows == 0) return HB_OK;
    AdaParams p{x, y, gate, shift, scale, x_out, h_out, x_rs, y_rs, xo_rs, h_rs, mod_bs, rows, rows_per_batch, C, eps};
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    return dtype == 1 ? launch_adaln<true>(p, st) : launch_adaln<false>(p, st);
}
