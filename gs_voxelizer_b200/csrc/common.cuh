// Shared definitions of the sm_100a voxelization kernels.
#pragma once

#include <algorithm>
#include <climits>
#include <cstdint>
#include <cuda_runtime.h>

namespace gsv {

// Tile edge in voxels, fixed by the reference's binning format
// (gs_voxelizer/cuda/config.h:1-4): tile ids and tile_bins depend on it.
constexpr int kTile = 8;
constexpr int kTileVoxels = kTile * kTile * kTile;
constexpr int kMaxChannels = 4;
constexpr int kSMs = 148;

// Geometry of the volume, or of a z-slab of it, as the kernels see it.
// The full volume is the slab [0, Tz).
struct Geom {
    int X, Y, Z;        // full-volume voxel extents
    int Tx, Ty, Tz;     // full-volume tile extents
    int tz0, tz1;       // tile-z range of the slab
    __host__ __device__ int slab_tiles_z() const { return tz1 - tz0; }
    __host__ __device__ int64_t slab_tiles() const {
        return (int64_t)(tz1 - tz0) * Ty * Tx;
    }
    // voxel z range of the slab's output buffer
    __host__ __device__ int z_begin() const { return tz0 * kTile; }
    __host__ __device__ int z_end() const { return min(Z, tz1 * kTile); }
};

inline Geom make_geom(const int32_t vol_zyx[3], int tz0 = 0, int tz1 = -1) {
    Geom g;
    g.Z = vol_zyx[0];
    g.Y = vol_zyx[1];
    g.X = vol_zyx[2];
    g.Tx = (g.X + kTile - 1) / kTile;
    g.Ty = (g.Y + kTile - 1) / kTile;
    g.Tz = (g.Z + kTile - 1) / kTile;
    g.tz0 = tz0;
    g.tz1 = tz1 < 0 ? g.Tz : tz1;
    return g;
}

// Running count of kernels this library has launched (gsv_launch_count()).
void count_launches(int k);

// Blocks of the tile scans (binning, backward plan) for ntiles tiles; the
// scans leave their grand total at partials[scan_blocks(ntiles)].
long long scan_blocks(long long ntiles);

// The per-Gaussian backward's work plan, built while binning (fused-L1
// forward): per-tile work-item ranges `item_bins` (int2 per tile), the scan
// partials of the item counts (total in partials[scan_blocks(ntiles)]), the
// item descriptors (tile, first pair, Gaussians) and the item buffer's
// capacity, to which ranges are clamped.
struct ItemScan {
    long long *partials;
    int *item_bins;
    int4 *desc;
    long long cap;
};

// Inputs of the tensor-core backward (one channel, fused L1) that the fused
// forward leaves in the workspace: the per-tile sign plane, the tile of every
// pair and the binning's pair total.
struct TcInputs {
    const float *sign_plane;
    const int *tile_of;
    const long long *pair_total;
};

// Normalised 11-tap Gaussian window of the 3D SSIM (host copy, ssim.cu).
struct SsWindowHost {
    float w[11];
};

// Stages of launch_vox_backward_gauss: everything, or only the kernel (the
// fused-L1 forward left the records and the work plan in the workspace).
enum BwdStage { kBwdFull = 0, kBwdPrepared = 2 };

// Optional CUDA events recorded right before / after the main voxelization
// kernels (gsv_profile_kernel()); no-ops unless a caller installed events.
enum ProfKind { kProfForward = 0, kProfBackwardGauss = 1, kProfBackwardVoxel = 2 };
void profile_mark(int kind, bool stop, cudaStream_t stream);

// Halo exchange of owner-sharded Gaussians (halo.cu): record sizes in
// floats and the per-call description of the peers, passed to the kernels
// by value.
constexpr int kHaloMaxRanks = 64;
constexpr int kHaloRec = 20;   // render record: pr 4, conic 6, I 4, tile box 6
constexpr int kHaloGrad = 16;  // gradient record: pr 4, conic 6, I 4, pad 2
struct HaloPeers {
    int world, rank;
    int tz0[kHaloMaxRanks], tz1[kHaloMaxRanks];  // tile-z range of each slab
    long long off[kHaloMaxRanks];                // segment start (records)
    int cap[kHaloMaxRanks];                      // slots per segment
    long long loff[kHaloMaxRanks];               // local index of slot 0 - n_own
    // where this rank's segment for peer d starts (its header record): in a
    // local send buffer, or directly in peer d's receive buffer (its device
    // memory, reached over NVLink); the packing kernels write there
    float *dst[kHaloMaxRanks];
};

// 2^x on the special-function unit (MUFU.EX2), flush-to-zero.
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Paired FP32 multiply / FMA with flush-to-zero (FMUL2.FTZ / FFMA2.FTZ):
// a result below the smallest normal float is exactly 0.
__device__ __forceinline__ float2 fmul2_ftz(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\t"
        "mov.b64 rb, {%4, %5};\n\t"
        "mul.rn.ftz.f32x2 rd, ra, rb;\n\t"
        "mov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

__device__ __forceinline__ float2 ffma2_ftz(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\t"
        "mov.b64 rb, {%4, %5};\n\t"
        "mov.b64 rc, {%6, %7};\n\t"
        "fma.rn.ftz.f32x2 rd, ra, rb, rc;\n\t"
        "mov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}

__device__ __forceinline__ unsigned lane_id() {
    unsigned l;
    asm("mov.u32 %0, %%laneid;" : "=r"(l));
    return l;
}

__device__ __forceinline__ int warp_inclusive_scan(int v) {
    const unsigned lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= (unsigned)o) v += t;
    }
    return v;
}

__device__ __forceinline__ long long warp_inclusive_scan_ll(long long v) {
    const unsigned lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        long long t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= (unsigned)o) v += t;
    }
    return v;
}

__device__ __forceinline__ void red_add(float *p, float v) { atomicAdd(p, v); }
__device__ __forceinline__ void red_add2(float *p, float a, float b) {
    atomicAdd(reinterpret_cast<float2 *>(p), make_float2(a, b));
}
__device__ __forceinline__ void red_add4(float *p, float a, float b, float c,
                                         float d) {
    atomicAdd(reinterpret_cast<float4 *>(p), make_float4(a, b, c, d));
}

}  // namespace gsv
