// tinym_quant.cuh -- per-tensor E4M3 quantisation of the activation X: the
// prologue of the fused activation path (BF16 / FP32 X in, FP8 GEMM out).
//
// Restates the caller's step before the GEMM, the harness's
// quantize_per_tensor (fp8_gemm_task_harness.py:41-44):
//     scale = max(amax(|x|) / 448, 1e-12)            (FP32)
//     q     = e4m3_rne(clamp(x / scale, -448, 448))
// and alpha = scale * w_scale (harness make_case, :58).
//
// One thread-block cluster of kQuantCtas CTAs: each CTA takes a contiguous
// slice of X, reduces |x| to a local max, the cluster combines the maxima
// through distributed shared memory, and every CTA quantises its slice with
// the common scale.  Up to kQuantCtas * kQuantThreads * kQuantRegVecs * 16
// bytes of X (256 KiB: M = 16, K = 8192 in BF16) stay in registers between
// the two passes, so X is read from memory once; larger X is read twice.  The kernel releases the dependent GEMM
// (griddepcontrol.launch_dependents) on entry, so the GEMM's W stream runs
// while X is being quantised; the GEMM waits for this grid only before it
// loads X and alpha.
#pragma once

#include <cuda_fp8.h>

#include "tinym_ptx.cuh"

namespace tinym {

constexpr int kQuantCtas = 8;          // one (portable) cluster
constexpr int kQuantThreads = 512;
constexpr int kQuantRegVecs = 4;       // 16-byte vectors a thread keeps between the passes
constexpr int kQuantWsHeader = 256;    // workspace: f32 scale @0, f32 alpha @4, codes @256
constexpr float kE4m3Max = 448.0f;

// max(|a|, |b|) that propagates NaN like torch's amax.
__device__ __forceinline__ float nan_amax(float a, float b) {
    return (a != a || b != b) ? __int_as_float(0x7fc00000) : fmaxf(a, b);
}

__device__ __forceinline__ float dsmem_ld_f32(uint32_t cluster_addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(cluster_addr) : "memory");
    return v;
}

// 16 bytes of X -> N floats (exact widening).
template <typename T>
struct ActVec;
template <>
struct ActVec<__nv_bfloat16> {
    static constexpr int N = 8;
    __device__ __forceinline__ static void unpack(const uint4& u, float (&f)[8]) {
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            f[2 * i] = __uint_as_float(w[i] << 16);
            f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
        }
    }
};
template <>
struct ActVec<float> {
    static constexpr int N = 4;
    __device__ __forceinline__ static void unpack(const uint4& u, float (&f)[4]) {
        f[0] = __uint_as_float(u.x);
        f[1] = __uint_as_float(u.y);
        f[2] = __uint_as_float(u.z);
        f[3] = __uint_as_float(u.w);
    }
};

// clamp(x / scale, -448, 448) with torch's semantics (NaN passes through),
// then E4M3 round-to-nearest-even through the CUDA conversion intrinsic.
__device__ __forceinline__ uint32_t quant_pair(float a, float b, float scale) {
    float qa = __fdiv_rn(a, scale), qb = __fdiv_rn(b, scale);
    qa = qa > kE4m3Max ? kE4m3Max : (qa < -kE4m3Max ? -kE4m3Max : qa);
    qb = qb > kE4m3Max ? kE4m3Max : (qb < -kE4m3Max ? -kE4m3Max : qb);
    return static_cast<uint32_t>(
        __nv_cvt_float2_to_fp8x2(make_float2(qa, qb), __NV_SATFINITE, __NV_E4M3));
}

template <typename T>
__global__ void __cluster_dims__(kQuantCtas, 1, 1) __launch_bounds__(kQuantThreads)
    tinym_quant_act_kernel(const T* __restrict__ x, int64_t count, uint8_t* __restrict__ ws,
                           const float* __restrict__ w_scale) {
    grid_launch_dependents();  // the GEMM may start streaming W right away

    using V = ActVec<T>;
    __shared__ float s_warp[kQuantThreads / 32];
    __shared__ float s_amax;  // this CTA's max |x|, read by the whole cluster
    __shared__ float s_gmax;  // the cluster's max |x|

    const int64_t nvec = count / V::N;  // count % V::N == 0 (K % 16 == 0)
    const uint32_t rank = cluster_ctarank();
    const int64_t per = (nvec + kQuantCtas - 1) / kQuantCtas;
    const int64_t v0 = static_cast<int64_t>(rank) * per;
    const int64_t v1 = v0 + per < nvec ? v0 + per : nvec;
    const uint4* xv = reinterpret_cast<const uint4*>(x);

    // Pass 1: the first kQuantRegVecs vectors of this thread are loaded
    // together (independent loads in flight) and kept; the rest stream.
    uint4 keep[kQuantRegVecs];
    float m = 0.0f;
#pragma unroll
    for (int r = 0; r < kQuantRegVecs; ++r) {
        const int64_t v = v0 + threadIdx.x + static_cast<int64_t>(r) * kQuantThreads;
        keep[r] = v < v1 ? __ldg(xv + v) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int r = 0; r < kQuantRegVecs; ++r) {
        float f[V::N];
        V::unpack(keep[r], f);
#pragma unroll
        for (int j = 0; j < V::N; ++j) m = nan_amax(m, fabsf(f[j]));
    }
    for (int64_t v = v0 + threadIdx.x + static_cast<int64_t>(kQuantRegVecs) * kQuantThreads; v < v1;
         v += kQuantThreads) {
        float f[V::N];
        V::unpack(__ldg(xv + v), f);
#pragma unroll
        for (int j = 0; j < V::N; ++j) m = nan_amax(m, fabsf(f[j]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = nan_amax(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    if ((threadIdx.x & 31) == 0) s_warp[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float a = s_warp[0];
        for (int w = 1; w < kQuantThreads / 32; ++w) a = nan_amax(a, s_warp[w]);
        s_amax = a;
    }
    // Every CTA's local maximum is published before anyone reads it ...
    cluster_arrive_release();
    cluster_wait_acquire();
    // Lane r of warp 0 reads rank r's maximum (one remote latency in all),
    // the warp combines them, and the CTA takes the result from s_gmax.
    if (threadIdx.x < 32) {
        float a = threadIdx.x < kQuantCtas
                      ? dsmem_ld_f32(dsmem_map(smem_u32(&s_amax), threadIdx.x))
                      : 0.0f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a = nan_amax(a, __shfl_xor_sync(0xFFFFFFFFu, a, o));
        if (threadIdx.x == 0) s_gmax = a;
    }
    __syncthreads();
    const float amax = s_gmax;
    // ... and no CTA leaves while another may still read its s_amax.
    cluster_arrive_relaxed();

    float scale = __fdiv_rn(amax, kE4m3Max);
    scale = scale < 1e-12f ? 1e-12f : scale;  // clamp(min=1e-12); NaN stays NaN
    uint8_t* codes = ws + kQuantWsHeader;
    auto quantise = [&](int64_t v, const uint4& u) {
        float f[V::N];
        V::unpack(u, f);
        if constexpr (V::N == 8) {
            uint2 out;
            out.x = quant_pair(f[0], f[1], scale) | (quant_pair(f[2], f[3], scale) << 16);
            out.y = quant_pair(f[4], f[5], scale) | (quant_pair(f[6], f[7], scale) << 16);
            *reinterpret_cast<uint2*>(codes + v * 8) = out;
        } else {
            *reinterpret_cast<uint32_t*>(codes + v * 4) =
                quant_pair(f[0], f[1], scale) | (quant_pair(f[2], f[3], scale) << 16);
        }
    };
    // Pass 2: the kept vectors from registers, the rest read again.
#pragma unroll
    for (int r = 0; r < kQuantRegVecs; ++r) {
        const int64_t v = v0 + threadIdx.x + static_cast<int64_t>(r) * kQuantThreads;
        if (v < v1) quantise(v, keep[r]);
    }
    for (int64_t v = v0 + threadIdx.x + static_cast<int64_t>(kQuantRegVecs) * kQuantThreads; v < v1;
         v += kQuantThreads)
        quantise(v, __ldg(xv + v));
    if (rank == 0 && threadIdx.x == 0) {
        float* hdr = reinterpret_cast<float*>(ws);
        hdr[0] = scale;
        hdr[1] = scale * __ldg(w_scale);  // alpha, as (sa * sw).to(float32)
    }
    cluster_wait_acquire();
}

}  // namespace tinym
