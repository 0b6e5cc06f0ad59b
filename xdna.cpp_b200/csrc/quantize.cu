// Device-side synthetic weight generation for benchmarks and decode
// harnesses: N(0, sigma) F32 values from a counter-based generator and GPU
// quantisers to GGUF blocks.  A 70B-shaped Q4_K stack is 274 GB of F32 before
// quantisation, far too much to produce on the host, so it is generated and
// quantised layer by layer on the GPU.
//
// The quantisers use explicitly rounded IEEE operations (__fmul_rn etc., no
// contraction) so that they reproduce the CPU quantisers bit for bit:
//   Q4_0: ggml's quantize_row_q4_0_ref (the algorithm gguf/quants.py:220-238
//         restates): d = max / -8, q = min(15, (int)(x / d + 8.5));
//   Q4_K: an affine fit per 32-value sub-block (scale = (max - min) / 15,
//         min <= 0) with 6-bit scales and mins under fp16 d / dmin.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "formats.cuh"
#include "gemv.cuh"

namespace xb {
namespace {

__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__global__ void fill_normal_kernel(float* out, int64_t n, uint64_t seed, float sigma) {
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < (n + 1) / 2;
         i += int64_t(gridDim.x) * blockDim.x) {
        const uint64_t r = splitmix64(seed * 0x100000001B3ull + uint64_t(i));
        const float u1 = (float(uint32_t(r >> 40)) + 0.5f) * (1.0f / 16777216.0f);  // (0,1)
        const float u2 = float(uint32_t(r & 0xFFFFFFu)) * (1.0f / 16777216.0f);        // [0,1)
        const float rad = sigma * sqrtf(-2.0f * logf(u1));
        float s, c;
        sincospif(2.0f * u2, &s, &c);
        out[2 * i] = rad * c;
        if (2 * i + 1 < n) out[2 * i + 1] = rad * s;
    }
}

// one aligned 16-bit store (block offsets of Q4_0 / Q4_K are even)
__device__ __forceinline__ void st16(uint8_t* p, __half h) {
    *reinterpret_cast<unsigned short*>(p) = __half_as_ushort(h);
}

__global__ void quant_q4_0_kernel(const float* __restrict__ src, uint8_t* __restrict__ dst, int64_t nblocks) {
    for (int64_t ib = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; ib < nblocks; ib += int64_t(gridDim.x) * blockDim.x) {
        const float* x = src + ib * 32;
        uint8_t* b = dst + ib * 18;
        float amax = 0.f, maxv = 0.f;
        for (int j = 0; j < 32; ++j) {
            const float a = fabsf(x[j]);
            if (amax < a) {
                amax = a;
                maxv = x[j];
            }
        }
        const float d = __fdiv_rn(maxv, -8.0f);
        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        st16(b, __float2half_rn(d));
        for (int j = 0; j < 16; ++j) {
            int xi0 = __float2int_rz(__fadd_rn(__fmul_rn(x[j], id), 8.5f));
            int xi1 = __float2int_rz(__fadd_rn(__fmul_rn(x[16 + j], id), 8.5f));
            xi0 = min(15, max(0, xi0));
            xi1 = min(15, max(0, xi1));
            b[2 + j] = uint8_t(xi0 | (xi1 << 4));
        }
    }
}

__global__ void quant_q4_K_kernel(const float* __restrict__ src, uint8_t* __restrict__ dst, int64_t nblocks) {
    for (int64_t ib = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; ib < nblocks; ib += int64_t(gridDim.x) * blockDim.x) {
        const float* x = src + ib * 256;
        uint8_t* b = dst + ib * 144;
        float scale[8], minv[8];
        for (int j = 0; j < 8; ++j) {
            float mn = x[32 * j], mx = x[32 * j];
            for (int l = 1; l < 32; ++l) {
                const float v = x[32 * j + l];
                if (v < mn) mn = v;
                if (v > mx) mx = v;
            }
            if (mn > 0.0f) mn = 0.0f;
            scale[j] = __fdiv_rn(__fsub_rn(mx, mn), 15.0f);
            minv[j] = -mn;
        }
        float max_scale = 0.f, max_min = 0.f;
        for (int j = 0; j < 8; ++j) {
            if (scale[j] > max_scale) max_scale = scale[j];
            if (minv[j] > max_min) max_min = minv[j];
        }
        const float inv_scale = max_scale > 0.0f ? __fdiv_rn(63.0f, max_scale) : 0.0f;
        const float inv_min = max_min > 0.0f ? __fdiv_rn(63.0f, max_min) : 0.0f;
        int ls[8], lm[8];
        for (int j = 0; j < 8; ++j) {
            ls[j] = min(63, max(0, __float2int_rn(__fmul_rn(inv_scale, scale[j]))));
            lm[j] = min(63, max(0, __float2int_rn(__fmul_rn(inv_min, minv[j]))));
        }
        uint8_t s[12];
        for (int i = 0; i < 12; ++i) s[i] = 0;
        for (int j = 0; j < 8; ++j) {
            if (j < 4) {
                s[j] = uint8_t(ls[j] & 63);
                s[j + 4] = uint8_t(lm[j] & 63);
            } else {
                s[j + 4] = uint8_t((ls[j] & 0x0f) | ((lm[j] & 0x0f) << 4));
                s[j - 4] = uint8_t(s[j - 4] | ((ls[j] >> 4) << 6));
                s[j] = uint8_t(s[j] | ((lm[j] >> 4) << 6));
            }
        }
        const __half dh = __float2half_rn(__fdiv_rn(max_scale, 63.0f));
        const __half dmh = __float2half_rn(__fdiv_rn(max_min, 63.0f));
        st16(b, dh);
        st16(b + 2, dmh);
        for (int i = 0; i < 12; ++i) b[4 + i] = s[i];
        const float dd = __half2float(dh), dm = __half2float(dmh);
        uint8_t L[256];
        for (int j = 0; j < 8; ++j) {
            const float sc = __fmul_rn(dd, float(ls[j]));
            const float m = __fmul_rn(dm, float(lm[j]));
            for (int l = 0; l < 32; ++l) {
                const int q = sc > 0.0f ? __float2int_rn(__fdiv_rn(__fadd_rn(x[32 * j + l], m), sc)) : 0;
                L[32 * j + l] = uint8_t(min(15, max(0, q)));
            }
        }
        for (int j = 0; j < 4; ++j)
            for (int l = 0; l < 32; ++l) b[16 + 32 * j + l] = uint8_t(L[64 * j + l] | (L[64 * j + 32 + l] << 4));
    }
}

unsigned grid_for(int64_t n, int threads) {
    const int64_t b = (n + threads - 1) / threads;
    return unsigned(b < 1 ? 1 : (b > 65536 ? 65536 : b));
}

}  // namespace

bool quantize_supported(int type) { return type == T_Q4_0 || type == T_Q4_K; }

cudaError_t fill_normal_launch(float* out, int64_t n, uint64_t seed, float sigma, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    fill_normal_kernel<<<grid_for((n + 1) / 2, 256), 256, 0, stream>>>(out, n, seed, sigma);
    return cudaGetLastError();
}

cudaError_t quantize_launch(int type, const float* src, void* dst, int64_t N, int64_t K, cudaStream_t stream) {
    const FormatInfo f = format_info(type);
    if (!quantize_supported(type) || K % f.block_vals || N < 0) return cudaErrorInvalidValue;
    const int64_t nblocks = N * (K / f.block_vals);
    if (nblocks == 0) return cudaSuccess;
    if (type == T_Q4_0)
        quant_q4_0_kernel<<<grid_for(nblocks, 128), 128, 0, stream>>>(src, static_cast<uint8_t*>(dst), nblocks);
    else
        quant_q4_K_kernel<<<grid_for(nblocks, 128), 128, 0, stream>>>(src, static_cast<uint8_t*>(dst), nblocks);
    return cudaGetLastError();
}

}  // namespace xb
