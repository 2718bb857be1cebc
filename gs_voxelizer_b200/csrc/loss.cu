// L1 loss between a voxelized volume and a target volume, and its gradient.
//
// Not part of the reference's extension: the reference's own benchmarks and
// its users compute losses in PyTorch (test/compare_speed.py uses a 3D SSIM).
// The L1 loss here is the one the training-step benchmark uses; it exists
// standalone (two HBM-bound passes) and fused into the voxelization kernels
// (the forward kernel reduces |vol - target| per tile as it stores the
// volume, and the backward kernel forms sign(vol - target) while staging
// each tile, so dL/dvol is never written to HBM).
//
// Reductions are deterministic: fixed grid for a given size, per-block sums
// in double, then one block summing the partials in order (one block alone
// for up to 64K elements).
#include "common.cuh"

namespace gsv {
namespace {

constexpr int kRedThreads = 256;

__device__ __forceinline__ double block_sum_d(double v, double *smem) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) smem[wid] = v;
    __syncthreads();
    double t = 0.0;
    if (wid == 0) {
        t = lane < (int)(blockDim.x >> 5) ? smem[lane] : 0.0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
            t += __shfl_xor_sync(0xffffffffu, t, o);
    }
    return t;  // valid in thread 0
}

// partial[b] = sum over this block's share of |a - b| (or of a if b null)
__global__ void __launch_bounds__(kRedThreads)
abs_diff_partials_kernel(long long n, const float *__restrict__ a,
                         const float *__restrict__ b,
                         double *__restrict__ partial) {
    __shared__ double smem[32];
    const long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long stride = (long long)gridDim.x * blockDim.x;
    float s = 0.f;
    const bool vec = ((reinterpret_cast<uintptr_t>(a) |
                       reinterpret_cast<uintptr_t>(b)) & 15) == 0;
    if (vec) {
        const long long n4 = n / 4;
        const float4 *a4 = reinterpret_cast<const float4 *>(a);
        const float4 *b4 = reinterpret_cast<const float4 *>(b);
        for (long long i = tid; i < n4; i += stride) {
            const float4 x = __ldg(a4 + i);
            if (b) {
                const float4 y = __ldg(b4 + i);
                s += fabsf(x.x - y.x) + fabsf(x.y - y.y) + fabsf(x.z - y.z) +
                     fabsf(x.w - y.w);
            } else {
                s += x.x + x.y + x.z + x.w;
            }
        }
        for (long long i = 4 * n4 + tid; i < n; i += stride)
            s += b ? fabsf(a[i] - b[i]) : a[i];
    } else {
        for (long long i = tid; i < n; i += stride)
            s += b ? fabsf(a[i] - b[i]) : a[i];
    }
    const double t = block_sum_d((double)s, smem);
    if (threadIdx.x == 0) partial[blockIdx.x] = t;
}

// out[0] = (float)(sum(partial) * inv_denom), summed in index order
__global__ void __launch_bounds__(kRedThreads)
finish_sum_kernel(const double *__restrict__ partial, int nparts,
                  double inv_denom, float *__restrict__ out) {
    __shared__ double smem[32];
    double s = 0.0;
    const int per = (nparts + kRedThreads - 1) / kRedThreads;
    for (int k = 0; k < per; ++k) {
        const int i = threadIdx.x * per + k;
        if (i < nparts) s += partial[i];
    }
    const double t = block_sum_d(s, smem);
    if (threadIdx.x == 0) out[0] = (float)(t * inv_denom);
}

// Small inputs: one CTA of 1024 threads, thread t summing elements t,
// t + 1024, ... in order (coalesced), then a block sum: out[0] = sum *
// inv_denom in one launch.
constexpr int kSmallSumThreads = 1024;
constexpr long long kSmallSum = 64 * 1024;

__global__ void __launch_bounds__(kSmallSumThreads)
sum_small_kernel(long long n, const float *__restrict__ a,
                 const float *__restrict__ b, double inv_denom,
                 float *__restrict__ out) {
    __shared__ double smem[32];
    float s = 0.f;
    if (b) {
#pragma unroll 8
        for (long long i = threadIdx.x; i < n; i += kSmallSumThreads)
            s += fabsf(a[i] - b[i]);
    } else {
#pragma unroll 8
        for (long long i = threadIdx.x; i < n; i += kSmallSumThreads)
            s += a[i];
    }
    const double t = block_sum_d((double)s, smem);
    if (threadIdx.x == 0) out[0] = (float)(t * inv_denom);
}

// grad = sign(vol - target) * (*grad_loss) * inv_denom
__global__ void __launch_bounds__(kRedThreads)
l1_grad_kernel(long long n, const float *__restrict__ vol,
               const float *__restrict__ target,
               const float *__restrict__ grad_loss, float inv_denom,
               float *__restrict__ grad) {
    const float k = (*grad_loss) * inv_denom;
    const long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long stride = (long long)gridDim.x * blockDim.x;
    auto sgn = [k](float d) { return d > 0.f ? k : (d < 0.f ? -k : 0.f); };
    const bool vec = ((reinterpret_cast<uintptr_t>(vol) |
                       reinterpret_cast<uintptr_t>(target) |
                       reinterpret_cast<uintptr_t>(grad)) & 15) == 0;
    long long done = 0;
    if (vec) {
        const long long n4 = n / 4;
        for (long long i = tid; i < n4; i += stride) {
            const float4 v = __ldg(reinterpret_cast<const float4 *>(vol) + i);
            const float4 t = __ldg(reinterpret_cast<const float4 *>(target) + i);
            reinterpret_cast<float4 *>(grad)[i] =
                make_float4(sgn(v.x - t.x), sgn(v.y - t.y), sgn(v.z - t.z),
                            sgn(v.w - t.w));
        }
        done = 4 * n4;
    }
    for (long long i = done + tid; i < n; i += stride)
        grad[i] = sgn(vol[i] - target[i]);
}

int reduce_blocks(long long n) {
    const long long want = (n + kRedThreads * 16 - 1) / (kRedThreads * 16);
    return (int)std::max<long long>(1, std::min<long long>(want, kSMs * 8));
}

}  // namespace

size_t l1_workspace_bytes(long long n) {
    return sizeof(double) * (size_t)reduce_blocks(n);
}

// out[0] = sum(a) * inv_denom (b == nullptr) or sum|a - b| * inv_denom
cudaError_t launch_sum(long long n, const float *a, const float *b,
                       double inv_denom, float *out, void *ws,
                       cudaStream_t stream) {
    if (n <= kSmallSum) {
        sum_small_kernel<<<1, kSmallSumThreads, 0, stream>>>(n, a, b,
                                                             inv_denom, out);
        count_launches(1);
        return cudaGetLastError();
    }
    const int blocks = reduce_blocks(n);
    double *partial = static_cast<double *>(ws);
    abs_diff_partials_kernel<<<blocks, kRedThreads, 0, stream>>>(n, a, b,
                                                                  partial);
    finish_sum_kernel<<<1, kRedThreads, 0, stream>>>(partial, blocks,
                                                     inv_denom, out);
    count_launches(2);
    return cudaGetLastError();
}

cudaError_t launch_l1_grad(long long n, const float *vol, const float *target,
                           const float *grad_loss, float inv_denom,
                           float *grad, cudaStream_t stream) {
    const long long want = (n / 4 + kRedThreads - 1) / kRedThreads;
    const int blocks =
        (int)std::max<long long>(1, std::min<long long>(want, kSMs * 16));
    l1_grad_kernel<<<blocks, kRedThreads, 0, stream>>>(n, vol, target,
                                                       grad_loss, inv_denom,
                                                       grad);
    count_launches(1);
    return cudaGetLastError();
}

}  // namespace gsv
