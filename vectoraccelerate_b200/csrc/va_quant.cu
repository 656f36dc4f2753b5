// va_quant.cu -- scalar (int8/int4) and binary quantization on the device. HBM-bound elementwise
// work: grid-stride loops over 16-byte vectors, grids sized to a multiple of the SM count.
//
// Scalar: quantize_int8_kernel / dequantize_int8_kernel / quantize_int4_kernel /
// dequantize_int4_kernel (Metal/Shaders/DataTransformations.metal:142-306). Parameters follow
// ScalarQuantizationKernel.computeQuantizationParams (ScalarQuantizationKernel.swift:496-520),
// computed by the caller from va_minmax. rint = round half to even, like Metal's rint.
// Binary: binaryQuantize (Metal/Shaders/QuantizationShaders.metal:132-160), LSB-first words.
#include <cfloat>

#include "va_internal.cuh"

namespace {

struct SqParams {
    float scale;
    int8_t zp;
    const float* scales;
    const int8_t* zps;
    int64_t per_channel;  // elements per channel (0 = global)
    int64_t n_channels;
};

__device__ __forceinline__ void sq_param(const SqParams& p, int64_t i, float& s, int8_t& z) {
    s = p.scale;
    z = p.zp;
    if (p.scales && p.per_channel > 0) {
        int64_t c = i / p.per_channel;
        if (c < p.n_channels) {
            s = p.scales[c];
            z = p.zps ? p.zps[c] : (int8_t)0;
        }
    }
}

__device__ __forceinline__ int8_t q8(float v, float s, int8_t z) {
    if (fabsf(s) < 1e-9f) return z;
    float r = rintf(__fdiv_rn(v, s) + (float)z);
    r = fminf(127.f, fmaxf(-128.f, r));
    return (int8_t)r;
}

__global__ void k_sq_q8(const float* __restrict__ x, int64_t n, SqParams p, int8_t* __restrict__ out) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        float s;
        int8_t z;
        sq_param(p, i, s, z);
        out[i] = q8(x[i], s, z);
    }
}

__global__ void k_sq_dq8(const int8_t* __restrict__ in, int64_t n, SqParams p, float* __restrict__ out) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        float s;
        int8_t z;
        sq_param(p, i, s, z);
        out[i] = ((float)in[i] - (float)z) * s;
    }
}

__global__ void k_sq_q4(const float* __restrict__ x, int64_t n, float s, int8_t z, uint8_t* __restrict__ out) {
    int64_t nb = (n + 1) / 2;
    for (int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; b < nb; b += (int64_t)gridDim.x * blockDim.x) {
        int64_t i0 = 2 * b, i1 = i0 + 1;
        float v0 = x[i0], v1 = i1 < n ? x[i1] : 0.f;
        float r0 = fabsf(s) < 1e-9f ? (float)z : __fdiv_rn(v0, s) + (float)z;
        float r1 = fabsf(s) < 1e-9f ? (float)z : __fdiv_rn(v1, s) + (float)z;
        int q0 = (int)fminf(7.f, fmaxf(-8.f, rintf(r0)));
        int q1 = (int)fminf(7.f, fmaxf(-8.f, rintf(r1)));
        out[b] = (uint8_t)(((q1 & 0xF) << 4) | (q0 & 0xF));
    }
}

__global__ void k_sq_dq4(const uint8_t* __restrict__ in, int64_t n, float s, int8_t z, float* __restrict__ out) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        uint8_t byte = in[i / 2];
        int nib = (i & 1) ? (byte >> 4) : (byte & 0xF);
        int q = (nib & 8) ? nib - 16 : nib;
        out[i] = ((float)q - (float)z) * s;
    }
}

__global__ void k_minmax(const float* __restrict__ x, int64_t n, unsigned* __restrict__ out_keys) {
    float mn = INFINITY, mx = -INFINITY;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        float v = x[i];
        mn = fminf(mn, v);
        mx = fmaxf(mx, v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        mn = fminf(mn, __shfl_xor_sync(0xFFFFFFFFu, mn, o));
        mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
    }
    if ((threadIdx.x & 31) == 0) {
        atomicMin(&out_keys[0], va::f2key(mn));
        atomicMax(&out_keys[1], va::f2key(mx));
    }
}

__global__ void k_keys_to_floats(unsigned* keys, float* out) {
    if (threadIdx.x == 0) {
        out[0] = va::key2f(keys[0]);
        out[1] = va::key2f(keys[1]);
    }
}

__global__ void k_init_minmax(unsigned* keys) {
    if (threadIdx.x == 0) {
        keys[0] = 0xFFFFFFFFu;
        keys[1] = 0u;
    }
}

// One warp per (row, 32-dimension word): lane b tests dimension 32w + b; the ballot is the word,
// LSB = lowest dimension (QuantizationShaders.metal:143-159).
__global__ void k_binary_quantize(const float* __restrict__ x, int64_t n, int dim, float threshold,
                                  uint32_t* __restrict__ out) {
    const int words = (dim + 31) / 32;
    const int64_t total = n * words;
    const int lane = threadIdx.x & 31;
    for (int64_t wi = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; wi < total;
         wi += ((int64_t)gridDim.x * blockDim.x) >> 5) {
        int64_t r = wi / words;
        int w = (int)(wi % words);
        int d = w * 32 + lane;
        bool bit = d < dim && x[r * dim + d] > threshold;
        uint32_t word = __ballot_sync(0xFFFFFFFFu, bit);
        if (lane == 0) out[wi] = word;
    }
}

int grid_for(va_context* ctx, int64_t work, int threads) {
    int64_t b = (work + threads - 1) / threads;
    int64_t cap = (int64_t)ctx->sm_count * 8;
    return (int)std::max<int64_t>(1, std::min(b, cap));
}

}  // namespace

extern "C" {

int va_sq_quantize_int8(va_context* ctx, const float* x, int64_t n, float scale, int8_t zero_point, const float* scales,
                        const int8_t* zps, int64_t n_channels, int8_t* out) {
    VA_REQUIRE(ctx && x && out, "ctx, x and out must not be NULL");
    VA_REQUIRE(n > 0, "numElements must be positive, got %lld", (long long)n);
    VA_REQUIRE(!scales || n_channels > 0, "n_channels must be positive with per-channel scales");
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    SqParams p{scale, zero_point, scales, zps, scales ? n / n_channels : 0, n_channels};
    k_sq_q8<<<grid_for(ctx, n, 256), 256, 0, ctx->stream>>>(x, n, p, out);
    return va_check_launch("k_sq_q8");
}

int va_sq_dequantize_int8(va_context* ctx, const int8_t* in, int64_t n, float scale, int8_t zero_point,
                          const float* scales, const int8_t* zps, int64_t n_channels, float* out) {
    VA_REQUIRE(ctx && in && out, "ctx, in and out must not be NULL");
    VA_REQUIRE(n > 0, "numElements must be positive, got %lld", (long long)n);
    VA_REQUIRE(!scales || n_channels > 0, "n_channels must be positive with per-channel scales");
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    SqParams p{scale, zero_point, scales, zps, scales ? n / n_channels : 0, n_channels};
    k_sq_dq8<<<grid_for(ctx, n, 256), 256, 0, ctx->stream>>>(in, n, p, out);
    return va_check_launch("k_sq_dq8");
}

int va_sq_quantize_int4(va_context* ctx, const float* x, int64_t n, float scale, int8_t zero_point, uint8_t* out) {
    VA_REQUIRE(ctx && x && out, "ctx, x and out must not be NULL");
    VA_REQUIRE(n > 0, "numElements must be positive, got %lld", (long long)n);
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    k_sq_q4<<<grid_for(ctx, (n + 1) / 2, 256), 256, 0, ctx->stream>>>(x, n, scale, zero_point, out);
    return va_check_launch("k_sq_q4");
}

int va_sq_dequantize_int4(va_context* ctx, const uint8_t* in, int64_t n, float scale, int8_t zero_point, float* out) {
    VA_REQUIRE(ctx && in && out, "ctx, in and out must not be NULL");
    VA_REQUIRE(n > 0, "numElements must be positive, got %lld", (long long)n);
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    k_sq_dq4<<<grid_for(ctx, n, 256), 256, 0, ctx->stream>>>(in, n, scale, zero_point, out);
    return va_check_launch("k_sq_dq4");
}

int va_minmax(va_context* ctx, const float* x, int64_t n, float* out_minmax) {
    VA_REQUIRE(ctx && x && out_minmax, "ctx, x and out_minmax must not be NULL");
    VA_REQUIRE(n > 0, "n must be positive, got %lld", (long long)n);
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    void* ws;
    VA_TRY(va_workspace(ctx, 2 * sizeof(unsigned), &ws));
    unsigned* keys = (unsigned*)ws;
    k_init_minmax<<<1, 32, 0, ctx->stream>>>(keys);
    k_minmax<<<grid_for(ctx, n, 256), 256, 0, ctx->stream>>>(x, n, keys);
    k_keys_to_floats<<<1, 32, 0, ctx->stream>>>(keys, out_minmax);
    return va_check_launch("k_minmax");
}

int va_binary_quantize(va_context* ctx, const float* x, int64_t n, int dim, float threshold, uint32_t* out) {
    VA_REQUIRE(ctx && x && out, "ctx, x and out must not be NULL");
    VA_REQUIRE(dim > 0, "dimension must be positive, got %d", dim);
    VA_REQUIRE(n >= 0, "n must be >= 0");
    if (!n) return VA_OK;
    VA_CUDA_TRY(cudaSetDevice(ctx->device));
    int64_t warps = n * ((dim + 31) / 32);
    k_binary_quantize<<<grid_for(ctx, warps * 32, 256), 256, 0, ctx->stream>>>(x, n, dim, threshold, out);
    return va_check_launch("k_binary_quantize");
}

}  // extern "C"
