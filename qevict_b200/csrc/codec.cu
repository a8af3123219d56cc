// Standalone codec entry points and shared host helpers.
#include <stdio.h>
#include <string.h>

#include "codec.cuh"

namespace qv {

static thread_local char g_cuda_err[256] = "";

int set_cuda_error(cudaError_t e) {
    snprintf(g_cuda_err, sizeof(g_cuda_err), "%s: %s", cudaGetErrorName(e), cudaGetErrorString(e));
    return QV_ECUDA;
}

int set_error_text(const char* msg) {
    snprintf(g_cuda_err, sizeof(g_cuda_err), "%s", msg);
    return QV_OK;
}

int check_launch() {
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? QV_OK : set_cuda_error(e);
}

size_t elt_size(int dt) { return dt == QV_F32 ? 4 : 2; }

int validate_dims(const qv_dims* d) {
    if (!d) return QV_EINVAL;
    if (d->batch <= 0 || d->kv_heads <= 0 || d->group <= 0 || d->group > 8) return QV_EINVAL;
    if (d->head_dim != 64 && d->head_dim != 128) return QV_EINVAL;
    if (d->omega < 16 || d->omega > 128 || d->omega % 16) return QV_EINVAL;
    if (d->sink < 0 || d->local < d->omega || d->local % d->omega) return QV_ENOTALIGNED;
    if (d->k_windows < 0 || d->q_windows < 0 || d->max_windows <= 0) return QV_EINVAL;
    if (d->k_windows + d->q_windows + 1 > 512) return QV_EINVAL;
    if (d->bits != 8 && d->bits != 4) return QV_EINVAL;
    if (d->dtype != QV_F32 && d->dtype != QV_BF16 && d->dtype != QV_F16) return QV_EINVAL;
    if (d->kv_heads > 32) return QV_EINVAL;
    return QV_OK;
}

template <int DT>
__global__ void __launch_bounds__(128) quantize_k_kernel(int om, int D, int bits, const void* x,
                                                         uint8_t* codes, void* s, void* z) {
    __shared__ float sm[256];
    const size_t w = blockIdx.x;
    const int qb = bits == 4 ? D / 2 : D;
    quantize_k_window<DT>(x, w * om * D, om, D, bits, false, codes, w * om * qb, s, z, w * D, false,
                          nullptr, nullptr, 0, sm);
}

template <int DT>
__global__ void __launch_bounds__(128) quantize_v_kernel(int om, int D, int bits, const void* x,
                                                         uint8_t* codes, void* s, void* z) {
    __shared__ float sm[256];
    const size_t w = blockIdx.x;
    const int qb = bits == 4 ? D / 2 : D;
    quantize_v_window<DT>(x, w * om * D, om, D, bits, false, codes, w * om * qb, s, z, w * om, false,
                          nullptr, nullptr, 0, sm);
}

template <int DT>
__global__ void __launch_bounds__(128) dequant_kernel(int om, int D, int bits, int per_token,
                                                      const uint8_t* codes, const void* s,
                                                      const void* z, void* out) {
    const size_t w = blockIdx.x;
    const int qb = bits == 4 ? D / 2 : D;
    for (int i = threadIdx.x; i < om * D; i += blockDim.x) {
        int t = i / D, d = i % D;
        uint32_t c = code_at(codes + (w * om + t) * qb, d, bits);
        size_t si = per_token ? w * om + t : w * D + d;
        st<DT>(out, w * om * D + i, dequant1<DT>(c, ld<DT>(s, si), ld<DT>(z, si)));
    }
}

static int codec_args_ok(int32_t n, int32_t om, int32_t D, int32_t bits, int32_t dt) {
    if (n < 0 || om <= 0 || om > 128 || (D != 64 && D != 128 && D != 16 && D != 32)) return QV_EINVAL;
    if (bits != 8 && bits != 4) return QV_EINVAL;
    if (dt != QV_F32 && dt != QV_BF16 && dt != QV_F16) return QV_EINVAL;
    return QV_OK;
}

}  // namespace qv

using namespace qv;

#define QV_DISPATCH_DT(dt, ...)                                   \
    switch (dt) {                                                 \
        case QV_F32: { constexpr int DT = QV_F32; __VA_ARGS__; } break;   \
        case QV_BF16: { constexpr int DT = QV_BF16; __VA_ARGS__; } break; \
        default: { constexpr int DT = QV_F16; __VA_ARGS__; } break;       \
    }

extern "C" int qv_quantize_k(int32_t n, int32_t om, int32_t D, int32_t bits, int32_t dt,
                             const void* x, uint8_t* codes, void* scale, void* zp, qv_stream_t stream) {
    int rc = codec_args_ok(n, om, D, bits, dt);
    if (rc) return rc;
    if (n == 0) return QV_OK;
    if (!x || !codes || !scale || !zp) return QV_EINVAL;
    QV_DISPATCH_DT(dt, quantize_k_kernel<DT><<<n, 128, 0, (cudaStream_t)stream>>>(om, D, bits, x, codes, scale, zp));
    return check_launch();
}

extern "C" int qv_quantize_v(int32_t n, int32_t om, int32_t D, int32_t bits, int32_t dt,
                             const void* x, uint8_t* codes, void* scale, void* zp, qv_stream_t stream) {
    int rc = codec_args_ok(n, om, D, bits, dt);
    if (rc) return rc;
    if (n == 0) return QV_OK;
    if (!x || !codes || !scale || !zp) return QV_EINVAL;
    QV_DISPATCH_DT(dt, quantize_v_kernel<DT><<<n, 128, 0, (cudaStream_t)stream>>>(om, D, bits, x, codes, scale, zp));
    return check_launch();
}

extern "C" int qv_dequantize(int32_t n, int32_t om, int32_t D, int32_t bits, int32_t dt, int32_t per_token,
                             const uint8_t* codes, const void* scale, const void* zp, void* out,
                             qv_stream_t stream) {
    int rc = codec_args_ok(n, om, D, bits, dt);
    if (rc) return rc;
    if (n == 0) return QV_OK;
    if (!codes || !scale || !zp || !out) return QV_EINVAL;
    QV_DISPATCH_DT(dt, dequant_kernel<DT><<<n, 128, 0, (cudaStream_t)stream>>>(om, D, bits, per_token, codes, scale, zp, out));
    return check_launch();
}

extern "C" int qv_read_error(const qv_layer* L, int32_t* host_err, qv_stream_t stream) {
    if (!L || !L->err || !host_err) return QV_EINVAL;
    cudaError_t e = cudaMemcpyAsync(host_err, L->err, sizeof(int32_t), cudaMemcpyDeviceToHost,
                                    (cudaStream_t)stream);
    if (e != cudaSuccess) return set_cuda_error(e);
    e = cudaStreamSynchronize((cudaStream_t)stream);
    if (e != cudaSuccess) return set_cuda_error(e);
    return QV_OK;
}

extern "C" const char* qv_last_cuda_error(void) { return g_cuda_err; }

extern "C" const char* qv_version(void) { return "qevict_b200 0.1 (sm_100a)"; }

extern "C" int32_t qv_ring_windows(const qv_dims* d) {
    if (validate_dims(d)) return -1;
    return d->local / d->omega + 1;
}

extern "C" int32_t qv_main_capacity(const qv_dims* d) {
    if (validate_dims(d)) return -1;
    return make_geo(d).S_cap;
}
