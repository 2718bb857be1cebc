// gsv_voxelize_forward_noalloc: the forward voxelization for callers that
// cannot allocate device memory.
//
// Some callers cannot hand this library a workspace: their device memory is
// owned by another allocator (a framework that reserves a GPU's memory up
// front), or they are host programs that receive only finished input and
// output buffers through a foreign-function interface and have no allocator
// of their own. The regular gsv_voxelize_forward needs a caller-provided
// workspace for its per-Gaussian render records; this variant keeps that
// scratch in a fixed array that lives in the library's own device image,
// so it allocates nothing at call time.
//
// Limits and rules:
//  * The scratch is kNoAllocScratchBytes (16 MiB) per GPU, held by every GPU
//    that loads the library until the process exits. It fits the records of
//    up to 16 MiB / (16 B * records per Gaussian) Gaussians: 349525 for 1-2
//    channels (48 B each), 262144 for 3-4 channels (64 B each). Larger
//    inputs are rejected with GSV_ERR_WORKSPACE_TOO_SMALL.
//  * All calls share the one array and it keeps the last call's contents.
//    Nothing in it needs to start at zero: each call rewrites every record it
//    reads before reading it. Calls whose kernels overlap on the GPU (for
//    example on two streams at once) race on the array; serialise them.
//  * The first call on a device looks up the array's device address with
//    cudaGetSymbolAddress (once per device, with that device current). Make
//    that first call before any stream capture.
#include <mutex>
#include <string>

#include "../../include/gsvox.h"
#include "common.cuh"

namespace gsv {
cudaError_t launch_vox_forward(const Geom &g, int C, int n, long long nisect,
                               const int *ids,
                               const int *tile_bins, const float *pos_radii,
                               const float *conics, const float *intens,
                               float *out, void *ws, cudaStream_t stream,
                               const float *target, float *loss_out,
                               double inv_denom);
void set_last_error(const char *msg);
}  // namespace gsv

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
constexpr int kMaxDevices = 64;

// Render-record scratch of the no-allocation forward. In host code this name
// is only a stand-in for the device array: its device address comes from
// cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char
    g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_setup_mutex;
void *g_scratch_ptr[kMaxDevices] = {};

// reports through gsv_last_error()
int noalloc_fail(int code, const std::string &msg) {
    gsv::set_last_error(msg.c_str());
    return code;
}

// Device address of the scratch array on the current device, looked up once.
cudaError_t scratch_address(void **out) {
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_ptr[dev]) {
        void *p = nullptr;
        err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (err != cudaSuccess) return err;
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return cudaSuccess;
}

}  // namespace

extern "C" {

int gsv_voxelize_forward_noalloc(const int32_t vol[3], int32_t C, int32_t n,
                                 int64_t nisect, const int32_t *ids,
                                 const int32_t *bins, const float *pos,
                                 const float *con, const float *inten,
                                 float *out, void *stream) {
    if (!vol || vol[0] <= 0 || vol[1] <= 0 || vol[2] <= 0)
        return noalloc_fail(GSV_ERR_INVALID_ARGUMENT,
                            "gsv_voxelize_forward_noalloc: bad vol_size_voxel");
    if (C < 1 || C > 4)
        return noalloc_fail(GSV_ERR_UNSUPPORTED_CHANNELS,
                            "gsv_voxelize_forward_noalloc: 1..4 channels supported");
    if (n < 0 || nisect < 0 || nisect > INT32_MAX)
        return noalloc_fail(GSV_ERR_INVALID_ARGUMENT,
                            "gsv_voxelize_forward_noalloc: bad sizes");
    const gsv::Geom g = gsv::make_geom(vol);
    if (g.slab_tiles() > INT32_MAX)
        return noalloc_fail(GSV_ERR_SIZE_OVERFLOW,
                            "gsv_voxelize_forward_noalloc: too many tiles");
    const size_t rec_bytes = (size_t)16 * (C <= 2 ? 3 : 4);
    const size_t max_n = kNoAllocScratchBytes / rec_bytes;
    if ((size_t)n > max_n)
        return noalloc_fail(
            GSV_ERR_WORKSPACE_TOO_SMALL,
            "gsv_voxelize_forward_noalloc: " + std::to_string(n) +
                " Gaussians exceed the fixed 16 MiB scratch (at most " +
                std::to_string(max_n) + " for " + std::to_string(C) +
                " channel(s)); use gsv_voxelize_forward with a workspace");
    const long long nvox = (long long)g.Z * g.Y * g.X * C;
    if (!out && nvox > 0)
        return noalloc_fail(GSV_ERR_INVALID_ARGUMENT,
                            "gsv_voxelize_forward_noalloc: out_vol is null");
    if (nisect > 0 && !(ids && bins && pos && con && inten))
        return noalloc_fail(GSV_ERR_INVALID_ARGUMENT,
                            "gsv_voxelize_forward_noalloc: null input pointer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t err;
    if (nisect == 0) {
        err = cudaMemsetAsync(out, 0, sizeof(float) * nvox, s);
    } else {
        void *scratch = nullptr;
        err = scratch_address(&scratch);
        if (err == cudaSuccess)
            err = gsv::launch_vox_forward(g, C, n, 0, ids, bins, pos, con, inten,
                                          out, scratch, s, nullptr, nullptr,
                                          1.0);
    }
    if (err != cudaSuccess)
        return noalloc_fail(GSV_ERR_CUDA,
                            std::string("gsv_voxelize_forward_noalloc: ") +
                                cudaGetErrorString(err));
    return GSV_OK;
}

}  // extern "C"
