// Q-cache codec device routines (block-cooperative, blockDim.x == 128).
//
// Bit-exact restatement of src/models/kv_cache/quantize.py:19-71 and of the
// path-C re-quantisation at src/models/kv_cache/quantize_manager.py:305-314:
// every torch op on the KV dtype is one fp32 op rounded to that dtype,
// torch.round is round-half-even (rintf), clamp then truncation to uint8.
#pragma once

#include "common.cuh"

namespace qv {

__device__ __forceinline__ float code_of(float ratio, float levels) {
    // torch.round(r).clamp(0, L).to(uint8); a NaN ratio (0/0 scale in fp16) maps to 0.
    if (ratio != ratio) return 0.f;
    float r = rintf(ratio);
    return fminf(fmaxf(r, 0.f), levels);
}

template <int DT>
__device__ __forceinline__ float scale_of(float mn, float mx, float levels) {
    // torch.clamp((t_max - t_min) / L, min=1e-8) in the KV dtype
    float s = div_r<DT>(sub_r<DT>(mx, mn), levels);
    return rnd<DT>(fmaxf(s, 1e-8f));
}

// Quantise one K window: x[t*xs + d] (t < om, d < D), per channel with RoPE-half
// tying.  zero_src: quantise an all-zero window instead of x (the reference's
// zero-filled gather, quantize_manager.py:256-258).  When use_meta is set the
// scale/zp are taken from (mks, mkz) instead of being derived (path C).
template <int DT>
__device__ void quantize_k_window(const void* x, size_t xbase, int om, int D, int bits, bool zero_src,
                                  uint8_t* codes, size_t cbase, void* ks, void* kz, size_t sbase,
                                  bool use_meta, const void* mks, const void* mkz, size_t mbase,
                                  float* smem /* >= 2*D floats */) {
    const float L = bits == 4 ? 15.f : 255.f;
    float* s_scale = smem;
    float* s_zp = smem + D;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float mn, mx;
        if (use_meta) {
            s_scale[d] = ld<DT>(mks, mbase + d);
            s_zp[d] = ld<DT>(mkz, mbase + d);
            continue;
        }
        if (zero_src) {
            mn = 0.f; mx = 0.f;
        } else {
            mn = INFINITY; mx = -INFINITY;
#pragma unroll 8
            for (int t = 0; t < om; ++t) {
                float v = ld<DT>(x, xbase + (size_t)t * D + d);
                mn = fminf(mn, v); mx = fmaxf(mx, v);
            }
        }
        s_scale[d] = mn;  // temporarily min
        s_zp[d] = mx;     // temporarily max
    }
    __syncthreads();
    if (!use_meta) {
        const int half = D / 2;
        float mn = 0.f, mx = 0.f;
        int d = threadIdx.x;
        if (d < half) {
            mn = fminf(s_scale[d], s_scale[d + half]);
            mx = fmaxf(s_zp[d], s_zp[d + half]);
        }
        __syncthreads();
        if (d < half) {
            float sc = scale_of<DT>(mn, mx, L);
            float zp = rnd<DT>(mn);
            s_scale[d] = sc; s_scale[d + half] = sc;
            s_zp[d] = zp; s_zp[d + half] = zp;
        }
        __syncthreads();
    }
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        st<DT>(ks, sbase + d, s_scale[d]);
        st<DT>(kz, sbase + d, s_zp[d]);
    }
    const int qb = bits == 4 ? D / 2 : D;
#pragma unroll 4
    for (int i = threadIdx.x; i < om * qb; i += blockDim.x) {
        int t = i / qb, j = i % qb;
        if (bits == 8) {
            float v = zero_src ? 0.f : ld<DT>(x, xbase + (size_t)t * D + j);
            float r = div_r<DT>(sub_r<DT>(v, s_zp[j]), s_scale[j]);
            codes[cbase + i] = (uint8_t)code_of(r, L);
        } else {
            int d0 = 2 * j, d1 = 2 * j + 1;
            float v0 = zero_src ? 0.f : ld<DT>(x, xbase + (size_t)t * D + d0);
            float v1 = zero_src ? 0.f : ld<DT>(x, xbase + (size_t)t * D + d1);
            uint32_t c0 = (uint32_t)code_of(div_r<DT>(sub_r<DT>(v0, s_zp[d0]), s_scale[d0]), L);
            uint32_t c1 = (uint32_t)code_of(div_r<DT>(sub_r<DT>(v1, s_zp[d1]), s_scale[d1]), L);
            codes[cbase + i] = (uint8_t)(((c0 << 4) | c1) & 0xFF);
        }
    }
    __syncthreads();
}

// Quantise one V window per token.  Scale/zp at vs/vz[sbase + t].
template <int DT>
__device__ void quantize_v_window(const void* x, size_t xbase, int om, int D, int bits, bool zero_src,
                                  uint8_t* codes, size_t cbase, void* vs, void* vz, size_t sbase,
                                  bool use_meta, const void* mvs, const void* mvz, size_t mbase,
                                  float* smem /* >= 2*om floats */) {
    const float L = bits == 4 ? 15.f : 255.f;
    float* s_scale = smem;
    float* s_zp = smem + om;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarp = blockDim.x >> 5;
    for (int t = warp; t < om; t += nwarp) {
        float sc, zp;
        if (use_meta) {
            sc = ld<DT>(mvs, mbase + t);
            zp = ld<DT>(mvz, mbase + t);
        } else {
            float mn = INFINITY, mx = -INFINITY;
            for (int d = lane; d < D; d += 32) {
                float v = zero_src ? 0.f : ld<DT>(x, xbase + (size_t)t * D + d);
                mn = fminf(mn, v); mx = fmaxf(mx, v);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            }
            sc = scale_of<DT>(mn, mx, L);
            zp = rnd<DT>(mn);
        }
        if (lane == 0) {
            s_scale[t] = sc; s_zp[t] = zp;
            st<DT>(vs, sbase + t, sc);
            st<DT>(vz, sbase + t, zp);
        }
    }
    __syncthreads();
    const int qb = bits == 4 ? D / 2 : D;
#pragma unroll 4
    for (int i = threadIdx.x; i < om * qb; i += blockDim.x) {
        int t = i / qb, j = i % qb;
        if (bits == 8) {
            float v = zero_src ? 0.f : ld<DT>(x, xbase + (size_t)t * D + j);
            codes[cbase + i] = (uint8_t)code_of(div_r<DT>(sub_r<DT>(v, s_zp[t]), s_scale[t]), L);
        } else {
            float v0 = zero_src ? 0.f : ld<DT>(x, xbase + (size_t)t * D + 2 * j);
            float v1 = zero_src ? 0.f : ld<DT>(x, xbase + (size_t)t * D + 2 * j + 1);
            uint32_t c0 = (uint32_t)code_of(div_r<DT>(sub_r<DT>(v0, s_zp[t]), s_scale[t]), L);
            uint32_t c1 = (uint32_t)code_of(div_r<DT>(sub_r<DT>(v1, s_zp[t]), s_scale[t]), L);
            codes[cbase + i] = (uint8_t)(((c0 << 4) | c1) & 0xFF);
        }
    }
    __syncthreads();
}

// code -> rnd(rnd(code * scale) + zp)   (quantize.py:62-71)
template <int DT>
__device__ __forceinline__ float dequant1(uint32_t code, float scale, float zp) {
    return add_r<DT>(mul_r<DT>((float)code, scale), zp);
}

__device__ __forceinline__ uint32_t code_at(const uint8_t* row, int d, int bits) {
    if (bits == 8) return row[d];
    uint32_t b = row[d >> 1];
    return (d & 1) ? (b & 0xF) : (b >> 4);
}

}  // namespace qv
