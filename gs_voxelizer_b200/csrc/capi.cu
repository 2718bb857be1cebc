// extern "C" entry points declared in include/gsvox.h: argument checks,
// workspace layout and dispatch to the kernels. No device allocation happens
// here; errors are returned as status codes with a per-thread message.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/gsvox.h"
#include "common.cuh"

namespace gsv {
cudaError_t launch_project_fwd(int n, int channels, const float *pos3d,
                               const float *scale3d, const float *quat,
                               const float *intensities, const int vol[3],
                               const float world[3], const float center[3],
                               float *pos_radii, float *conics, int *tile_min,
                               int *tile_max, int *num_tiles,
                               cudaStream_t stream);
cudaError_t launch_project_bwd(int n, const float *pos3d, const float *scale3d,
                               const float *quat, const int vol[3],
                               const float world[3], const float *pos_radii_grad,
                               const float *conics_grad, const float *pos_radii,
                               float *pos_grad, float *scale_grad,
                               float *quat_grad, cudaStream_t stream);
size_t bin_workspace_bytes(long long ntiles, long long nisect, long long n,
                           long long layers);
cudaError_t launch_binning(int n, long long nisect, const int *tmin,
                           const int *tmax, int Tx, int Ty, int tz0, int tz1,
                           int *ids_out, int *tile_bins, void *ws,
                           cudaStream_t stream, long long *count_out = nullptr,
                           float *overflow_out = nullptr,
                           const ItemScan *items = nullptr);
ItemScan vox_item_scan(void *ws, long long n, int C, long long ntiles,
                       long long nisect);
size_t halo_workspace_bytes(int n, int world);
cudaError_t launch_halo_pack(int n, int C, const float *pr, const float *cq,
                             const float *inten, const int *tmin,
                             const int *tmax, const HaloPeers &P,
                             int *slot_map, long long *counts_out, void *ws,
                             cudaStream_t stream);
cudaError_t launch_halo_unpack(int n_own, int C, const HaloPeers &R,
                               long long total_slots, const float *recv,
                               float *pr, float *cq, float *inten, int *tmin,
                               int *tmax, float *flags, cudaStream_t stream);
cudaError_t launch_halo_pack_grads(int n_own, int C, const HaloPeers &R,
                                   long long total_slots, const float *gp,
                                   const float *gc, const float *gi,
                                   const float *loss, const float *flags,
                                   cudaStream_t stream);
cudaError_t launch_halo_accumulate(int n, int C, const HaloPeers &P,
                                   const int *slot_map, const float *recv,
                                   float *gp, float *gc, float *gi,
                                   const float *loss, const float *flags,
                                   float *out, cudaStream_t stream);

cudaError_t launch_count_slab_pairs(int n, const int *tmin, const int *tmax,
                                    int tz0, int tz1, long long *out,
                                    cudaStream_t stream);
size_t vox_workspace_bytes(long long n, int channels, long long ntiles,
                           long long nisect);
cudaError_t launch_vox_forward(const Geom &g, int C, int n, long long nisect,
                               const int *ids,
                               const int *tile_bins, const float *pos_radii,
                               const float *conics, const float *intens,
                               float *out, void *ws, cudaStream_t stream,
                               const float *target, float *loss_out,
                               double inv_denom);
cudaError_t launch_vox_forward_ex(const Geom &g, int C, int n, long long nisect,
                                  const int *ids, const int *tile_bins,
                                  const float *pos_radii, const float *conics,
                                  const float *intens, float *out, void *ws,
                                  cudaStream_t stream, const float *target,
                                  float *loss_out, double inv_denom,
                                  float *sign_plane, int *tile_of);
cudaError_t launch_vox_backward_tc(const Geom &g, const int *ids,
                                   const int *tile_of, const float4 *rec,
                                   const float *sign_plane,
                                   const long long *pair_total,
                                   long long pair_cap, float *pos_grad,
                                   float *conic_grad, float *int_grad,
                                   const float *grad_loss, float inv_denom,
                                   cudaStream_t stream);
int tc_error_flag(bool clear);
int peer_error_flag(bool clear);
cudaError_t launch_peer_barrier(int world, int rank, const long long *sig_ptrs,
                                int *epoch, cudaStream_t stream);
SsWindowHost ssim_window(double sigma);
size_t ssim_workspace_bytes(int nch, int D, int H, int W);
cudaError_t launch_ssim_forward(int nch, int D, int H, int W, const float *img1,
                                const float *img2, float C1, float C2,
                                const SsWindowHost &w, float *ssim_out, void *ws,
                                cudaStream_t stream);
cudaError_t launch_ssim_backward(int nch, int D, int H, int W, const float *img1,
                                 const float *img2, const SsWindowHost &w,
                                 const float *grad_out, const void *ws,
                                 float *grad, cudaStream_t stream);
size_t tv_workspace_bytes(int nch, int D, int H, int W);
cudaError_t launch_tv(int nch, int D, int H, int W, const float *x, int iso,
                      float eps, float *value_out, const float *grad_out,
                      float *grad, void *ws, cudaStream_t stream);
cudaError_t launch_vox_backward_gauss(const Geom &g, int C, int n,
                                      long long nisect, const int *ids,
                                      const int *tile_bins,
                                      const float *pos_radii,
                                      const float *conics,
                                      const float *intens, const float *grad,
                                      float *pos_grad, float *conic_grad,
                                      float *int_grad, void *ws,
                                      cudaStream_t stream,
                                      const float *target,
                                      const float *grad_loss,
                                      float inv_denom, int stage,
                                      const TcInputs *tc = nullptr);
const long long *bin_pair_total(const void *ws, long long ntiles);
size_t l1_workspace_bytes(long long n);
cudaError_t launch_sum(long long n, const float *a, const float *b,
                       double inv_denom, float *out, void *ws,
                       cudaStream_t stream);
cudaError_t launch_l1_grad(long long n, const float *vol, const float *target,
                           const float *grad_loss, float inv_denom,
                           float *grad, cudaStream_t stream);
cudaError_t launch_empty_l1(long long nvox, const float *target,
                            double inv_denom, float *loss_out, void *ws,
                            cudaStream_t stream);
cudaError_t launch_vox_backward_voxel(const Geom &g, int C, int n,
                                      long long nisect, const int *ids,
                                      const int *tile_bins,
                                      const float *pos_radii,
                                      const float *conics,
                                      const float *intens, const float *grad,
                                      float *pos_grad, float *conic_grad,
                                      float *int_grad, void *ws,
                                      cudaStream_t stream);
void enable_large_smem();
}  // namespace gsv

namespace gsv {
static std::atomic<unsigned long long> g_launches{0};
void count_launches(int k) { g_launches.fetch_add((unsigned long long)k); }

static std::atomic<cudaEvent_t> g_prof[3][2] = {};
void profile_mark(int kind, bool stop, cudaStream_t stream) {
    cudaEvent_t e = g_prof[kind][stop ? 1 : 0].load();
    if (e) cudaEventRecord(e, stream);
}
}  // namespace gsv

namespace {

thread_local std::string g_last_error;

int fail(int code, const char *fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

}  // namespace

namespace gsv {
// Lets other translation units report through gsv_last_error().
void set_last_error(const char *msg) { g_last_error = msg; }
}  // namespace gsv

namespace {

int cuda_status(cudaError_t err, const char *where) {
    if (err == cudaSuccess) return GSV_OK;
    return fail(GSV_ERR_CUDA, "%s: CUDA error %d (%s)", where, (int)err,
                cudaGetErrorString(err));
}

bool check_vol(const int32_t v[3], const char *fn) {
    if (!v) {
        fail(GSV_ERR_INVALID_ARGUMENT, "%s: vol_size_voxel is null", fn);
        return false;
    }
    for (int i = 0; i < 3; ++i) {
        if (v[i] <= 0) {
            fail(GSV_ERR_INVALID_ARGUMENT,
                 "%s: vol_size_voxel must be positive, got (%d, %d, %d)", fn,
                 v[0], v[1], v[2]);
            return false;
        }
    }
    return true;
}

bool check_slab(const gsv::Geom &g, const char *fn) {
    if (g.tz0 < 0 || g.tz1 > g.Tz || g.tz0 > g.tz1) {
        fail(GSV_ERR_INVALID_ARGUMENT,
             "%s: tile z range [%d, %d) is outside [0, %d)", fn, g.tz0, g.tz1,
             g.Tz);
        return false;
    }
    return true;
}

#define GSV_REQUIRE(cond, code, ...)            \
    do {                                        \
        if (!(cond)) return fail(code, __VA_ARGS__); \
    } while (0)

cudaStream_t as_stream(void *s) { return static_cast<cudaStream_t>(s); }

int binning_impl(const char *fn, int32_t n, int64_t nisect,
                 const int32_t *tile_min, const int32_t *tile_max,
                 const gsv::Geom &g, int32_t *ids_out, int32_t *bins_out,
                 void *ws, size_t ws_bytes, void *stream) {
    GSV_REQUIRE(n >= 0 && nisect >= 0, GSV_ERR_INVALID_ARGUMENT,
                "%s: negative size (num_gaussians=%d, num_intersects=%lld)",
                fn, n, (long long)nisect);
    GSV_REQUIRE(nisect <= INT32_MAX, GSV_ERR_SIZE_OVERFLOW,
                "%s: num_intersects=%lld exceeds the int32 tile_bins format",
                fn, (long long)nisect);
    const long long ntiles = g.slab_tiles();
    GSV_REQUIRE(ntiles <= INT32_MAX, GSV_ERR_SIZE_OVERFLOW,
                "%s: %lld tiles exceed the int32 tile id format", fn, ntiles);
    GSV_REQUIRE(ntiles == 0 || bins_out, GSV_ERR_INVALID_ARGUMENT,
                "%s: tile_bins is null", fn);
    GSV_REQUIRE(nisect == 0 || (ids_out && tile_min && tile_max),
                GSV_ERR_INVALID_ARGUMENT, "%s: null input/output pointer", fn);
    const size_t need =
        gsv::bin_workspace_bytes(ntiles, nisect, n, g.slab_tiles_z());
    GSV_REQUIRE(ws_bytes >= need && (need == 0 || ws),
                GSV_ERR_WORKSPACE_TOO_SMALL,
                "%s: workspace of %zu bytes given, %zu needed", fn, ws_bytes,
                need);
    gsv::enable_large_smem();
    return cuda_status(gsv::launch_binning(n, nisect, tile_min, tile_max,
                                           g.Tx, g.Ty, g.tz0, g.tz1, ids_out,
                                           bins_out, ws, as_stream(stream)),
                       fn);
}

int vox_common_checks(const char *fn, const gsv::Geom &g, int32_t C,
                      int32_t n, int64_t nisect, const int32_t *ids,
                      const int32_t *bins, const float *pos, const float *con,
                      const float *inten, size_t ws_bytes, void *ws) {
    GSV_REQUIRE(C >= 1 && C <= 4, GSV_ERR_UNSUPPORTED_CHANNELS,
                "%s: %d channels requested, 1..4 supported", fn, C);
    GSV_REQUIRE(n >= 0 && nisect >= 0, GSV_ERR_INVALID_ARGUMENT,
                "%s: negative size", fn);
    GSV_REQUIRE(nisect <= INT32_MAX, GSV_ERR_SIZE_OVERFLOW,
                "%s: num_intersects exceeds int32", fn);
    GSV_REQUIRE(g.slab_tiles() <= INT32_MAX, GSV_ERR_SIZE_OVERFLOW,
                "%s: tile count exceeds int32", fn);
    if (nisect > 0) {
        GSV_REQUIRE(ids && bins && pos && con && inten,
                    GSV_ERR_INVALID_ARGUMENT, "%s: null input pointer", fn);
    }
    const size_t need =
        gsv::vox_workspace_bytes(n, C, g.slab_tiles(), nisect);
    GSV_REQUIRE(ws_bytes >= need && ws, GSV_ERR_WORKSPACE_TOO_SMALL,
                "%s: workspace of %zu bytes given, %zu needed", fn, ws_bytes,
                need);
    return GSV_OK;
}

int forward_impl(const char *fn, const gsv::Geom &g, int32_t C, int32_t n,
                 int64_t nisect, const int32_t *ids, const int32_t *bins,
                 const float *pos, const float *con, const float *inten,
                 float *out, void *ws, size_t ws_bytes, void *stream) {
    if (!check_slab(g, fn)) return GSV_ERR_INVALID_ARGUMENT;
    int st = vox_common_checks(fn, g, C, n, nisect, ids, bins, pos, con, inten,
                               ws_bytes, ws);
    if (st) return st;
    const long long nvox =
        (long long)(g.z_end() - g.z_begin()) * g.Y * g.X * C;
    GSV_REQUIRE(out || nvox == 0, GSV_ERR_INVALID_ARGUMENT, "%s: out_vol is null",
                fn);
    if (nisect == 0) {
        return cuda_status(cudaMemsetAsync(out, 0, sizeof(float) * nvox,
                                           as_stream(stream)),
                           fn);
    }
    return cuda_status(gsv::launch_vox_forward(g, C, n, nisect, ids, bins, pos, con,
                                               inten, out, ws,
                                               as_stream(stream), nullptr,
                                               nullptr, 1.0),
                       fn);
}

int backward_impl(const char *fn, bool per_gaussian, const gsv::Geom &g,
                  int32_t C, int32_t n, int64_t nisect, const int32_t *ids,
                  const int32_t *bins, const float *pos, const float *con,
                  const float *inten, const float *grad, float *pos_grad,
                  float *con_grad, float *int_grad, void *ws, size_t ws_bytes,
                  void *stream) {
    if (!check_slab(g, fn)) return GSV_ERR_INVALID_ARGUMENT;
    int st = vox_common_checks(fn, g, C, n, nisect, ids, bins, pos, con, inten,
                               ws_bytes, ws);
    if (st) return st;
    GSV_REQUIRE(n == 0 || (pos_grad && con_grad && int_grad),
                GSV_ERR_INVALID_ARGUMENT, "%s: null gradient output", fn);
    GSV_REQUIRE(nisect == 0 || grad, GSV_ERR_INVALID_ARGUMENT,
                "%s: vol_grad_in is null", fn);
    cudaError_t err =
        per_gaussian
            ? gsv::launch_vox_backward_gauss(g, C, n, nisect, ids, bins, pos,
                                             con, inten, grad, pos_grad,
                                             con_grad, int_grad, ws,
                                             as_stream(stream), nullptr,
                                             nullptr, 1.f, gsv::kBwdFull)
            : gsv::launch_vox_backward_voxel(g, C, n, nisect, ids, bins, pos,
                                             con, inten, grad, pos_grad,
                                             con_grad, int_grad, ws,
                                             as_stream(stream));
    return cuda_status(err, fn);
}

// Binning part of the fused-L1 workspace (256-byte aligned).
size_t l1_bin_part(const gsv::Geom &g, long long nisect, long long n) {
    return (gsv::bin_workspace_bytes(g.slab_tiles(), nisect, n,
                                     g.slab_tiles_z()) + 255) &
           ~size_t(255);
}

// Tensor-core backward inputs (one channel): the per-tile sign plane and
// the tile of every pair, after the binning and voxelization parts of the
// fused-L1 workspace.
bool g_use_tc_backward = false;

bool use_tc(int C) { return C == 1 && g_use_tc_backward; }

size_t l1_tc_part(const gsv::Geom &g, int C, long long nisect) {
    if (!use_tc(C)) return 0;
    return ((sizeof(float) * gsv::kTileVoxels * (size_t)g.slab_tiles() + 255) &
            ~size_t(255)) +
           ((sizeof(int) * (size_t)(nisect > 0 ? nisect : 1) + 255) & ~size_t(255));
}

struct TcBuffers {
    float *sign_plane;
    int *tile_of;
};

TcBuffers l1_tc_buffers(void *ws, const gsv::Geom &g, int C, int n,
                        long long nisect) {
    char *base = static_cast<char *>(ws) + l1_bin_part(g, nisect, n) +
                 gsv::vox_workspace_bytes(n, C, g.slab_tiles(), nisect);
    TcBuffers b;
    b.sign_plane = reinterpret_cast<float *>(base);
    b.tile_of = reinterpret_cast<int *>(
        base + ((sizeof(float) * gsv::kTileVoxels * (size_t)g.slab_tiles() + 255) &
                ~size_t(255)));
    return b;
}

// halo exchange: segment destinations, in a local send buffer (send + the
// segment's record offset) or given directly (seg_dst, device addresses in
// the peers' receive buffers); false if a needed one is missing
bool set_destinations(gsv::HaloPeers &P, float *send, const int64_t *seg_dst,
                      int rec) {
    for (int d = 0; d < P.world; ++d) {
        P.dst[d] = nullptr;
        if (d == P.rank) continue;
        if (seg_dst) {
            P.dst[d] = reinterpret_cast<float *>(static_cast<uintptr_t>(seg_dst[d]));
            if (!P.dst[d] || (seg_dst[d] & 15)) return false;
        } else {
            if (!send) return false;
            P.dst[d] = send + P.off[d] * rec;
        }
    }
    return true;
}

// halo exchange: per-peer description from the C arrays
bool make_peers(int32_t world, int32_t rank, const int32_t *slab_tz,
                const int64_t *seg_off, const int32_t *seg_slots,
                gsv::HaloPeers &P, long long &total_slots) {
    if (world < 1 || world > gsv::kHaloMaxRanks || rank < 0 || rank >= world ||
        !seg_off || !seg_slots)
        return false;
    P.world = world;
    P.rank = rank;
    long long loff = 0;
    for (int d = 0; d < world; ++d) {
        P.tz0[d] = slab_tz ? slab_tz[2 * d] : 0;
        P.tz1[d] = slab_tz ? slab_tz[2 * d + 1] : 0;
        P.off[d] = seg_off[d];
        P.cap[d] = d == rank ? 0 : seg_slots[d];
        if (P.cap[d] < 0 || P.off[d] < 0) return false;
        P.loff[d] = loff;
        loff += P.cap[d];
    }
    total_slots = loff;
    return true;
}

}  // namespace

extern "C" {

const char *gsv_last_error(void) { return g_last_error.c_str(); }

const char *gsv_version(void) { return "0.1.0"; }

uint64_t gsv_launch_count(void) { return gsv::g_launches.load(); }

int gsv_profile_kernel(int32_t which, void *start_event, void *stop_event) {
    GSV_REQUIRE(which >= 0 && which < 3, GSV_ERR_INVALID_ARGUMENT,
                "gsv_profile_kernel: which=%d not in 0..2", which);
    gsv::g_prof[which][0] = static_cast<cudaEvent_t>(start_event);
    gsv::g_prof[which][1] = static_cast<cudaEvent_t>(stop_event);
    return GSV_OK;
}

int gsv_optim_to_render_forward(int32_t n, int32_t C, const float *pos3d,
                                const float *scale3d, const float *quat,
                                const float *intensities,
                                const int32_t vol[3], const float world[3],
                                const float center[3], float *pos_radii,
                                float *conics, int32_t *tile_min,
                                int32_t *tile_max, int32_t *num_tiles,
                                void *stream) {
    const char *fn = "gsv_optim_to_render_forward";
    GSV_REQUIRE(C >= 1 && C <= 4, GSV_ERR_UNSUPPORTED_CHANNELS,
                "%s: %d channels requested, 1..4 supported", fn, C);
    GSV_REQUIRE(n >= 0, GSV_ERR_INVALID_ARGUMENT, "%s: negative size", fn);
    if (!check_vol(vol, fn)) return GSV_ERR_INVALID_ARGUMENT;
    GSV_REQUIRE(world && center, GSV_ERR_INVALID_ARGUMENT,
                "%s: null volume description", fn);
    if (n == 0) return GSV_OK;
    GSV_REQUIRE(pos3d && scale3d && quat && intensities && pos_radii &&
                    conics && tile_min && tile_max && num_tiles,
                GSV_ERR_INVALID_ARGUMENT, "%s: null pointer", fn);
    return cuda_status(
        gsv::launch_project_fwd(n, C, pos3d, scale3d, quat, intensities, vol,
                                world, center, pos_radii, conics, tile_min,
                                tile_max, num_tiles, as_stream(stream)),
        fn);
}

int gsv_optim_to_render_backward(int32_t n, const float *pos3d,
                                 const float *scale3d, const float *quat,
                                 const int32_t vol[3], const float world[3],
                                 const float center[3],
                                 const float *pos_radii_grad,
                                 const float *conics_grad,
                                 const float *pos_radii, float *pos_grad,
                                 float *scale_grad, float *quat_grad,
                                 void *stream) {
    const char *fn = "gsv_optim_to_render_backward";
    GSV_REQUIRE(n >= 0, GSV_ERR_INVALID_ARGUMENT, "%s: negative size", fn);
    if (!check_vol(vol, fn)) return GSV_ERR_INVALID_ARGUMENT;
    GSV_REQUIRE(world && center, GSV_ERR_INVALID_ARGUMENT,
                "%s: null volume description", fn);
    if (n == 0) return GSV_OK;
    GSV_REQUIRE(pos3d && scale3d && quat && pos_radii_grad && conics_grad &&
                    pos_radii && pos_grad && scale_grad && quat_grad,
                GSV_ERR_INVALID_ARGUMENT, "%s: null pointer", fn);
    return cuda_status(
        gsv::launch_project_bwd(n, pos3d, scale3d, quat, vol, world,
                                pos_radii_grad, conics_grad, pos_radii,
                                pos_grad, scale_grad, quat_grad,
                                as_stream(stream)),
        fn);
}

size_t gsv_bin_and_sort_workspace_bytes(int32_t n, int64_t nisect,
                                        const int32_t vol[3]) {
    if (!vol || vol[0] <= 0 || vol[1] <= 0 || vol[2] <= 0) return 0;
    const gsv::Geom g = gsv::make_geom(vol);
    return gsv::bin_workspace_bytes(g.slab_tiles(), nisect < 0 ? 0 : nisect,
                                    n < 0 ? 0 : n, g.slab_tiles_z());
}

int gsv_bin_and_sort_gaussians(int32_t n, int64_t nisect,
                               const int32_t *tile_min,
                               const int32_t *tile_max,
                               const int32_t *cum_tiles_hit,
                               const int32_t vol[3], int32_t *ids_out,
                               int32_t *bins_out, void *ws, size_t ws_bytes,
                               void *stream) {
    const char *fn = "gsv_bin_and_sort_gaussians";
    (void)cum_tiles_hit;
    if (!check_vol(vol, fn)) return GSV_ERR_INVALID_ARGUMENT;
    const gsv::Geom g = gsv::make_geom(vol);
    return binning_impl(fn, n, nisect, tile_min, tile_max, g, ids_out,
                        bins_out, ws, ws_bytes, stream);
}

size_t gsv_bin_and_sort_slab_workspace_bytes(int32_t n, int64_t nisect,
                                             const int32_t vol[3],
                                             int32_t tz0, int32_t tz1) {
    if (!vol || vol[0] <= 0 || vol[1] <= 0 || vol[2] <= 0) return 0;
    const gsv::Geom g = gsv::make_geom(vol, tz0, tz1);
    if (g.tz0 < 0 || g.tz1 > g.Tz || g.tz0 > g.tz1) return 0;
    return gsv::bin_workspace_bytes(g.slab_tiles(), nisect < 0 ? 0 : nisect,
                                    n < 0 ? 0 : n, g.slab_tiles_z());
}

int gsv_bin_and_sort_gaussians_slab(int32_t n, int64_t nisect,
                                    const int32_t *tile_min,
                                    const int32_t *tile_max,
                                    const int32_t vol[3], int32_t tz0,
                                    int32_t tz1, int32_t *ids_out,
                                    int32_t *bins_out, void *ws,
                                    size_t ws_bytes, void *stream) {
    const char *fn = "gsv_bin_and_sort_gaussians_slab";
    if (!check_vol(vol, fn)) return GSV_ERR_INVALID_ARGUMENT;
    const gsv::Geom g = gsv::make_geom(vol, tz0, tz1);
    if (!check_slab(g, fn)) return GSV_ERR_INVALID_ARGUMENT;
    return binning_impl(fn, n, nisect, tile_min, tile_max, g, ids_out,
                        bins_out, ws, ws_bytes, stream);
}

int gsv_count_slab_intersects(int32_t n, const int32_t *tile_min,
                              const int32_t *tile_max, int32_t tz0,
                              int32_t tz1, int64_t *count_out, void *stream) {
    const char *fn = "gsv_count_slab_intersects";
    GSV_REQUIRE(n >= 0 && tz0 >= 0 && tz1 >= tz0, GSV_ERR_INVALID_ARGUMENT,
                "%s: bad arguments", fn);
    GSV_REQUIRE(count_out && (n == 0 || (tile_min && tile_max)),
                GSV_ERR_INVALID_ARGUMENT, "%s: null pointer", fn);
    return cuda_status(
        gsv::launch_count_slab_pairs(n, tile_min, tile_max, tz0, tz1,
                                     reinterpret_cast<long long *>(count_out),
                                     as_stream(stream)),
        fn);
}

size_t gsv_voxelize_workspace_bytes(int32_t n, int32_t C, int64_t nisect,
                                    const int32_t vol[3]) {
    if (!vol || vol[0] <= 0 || vol[1] <= 0 || vol[2] <= 0) return 0;
    if (C < 1 || C > 4) return 0;
    const gsv::Geom g = gsv::make_geom(vol);
    return gsv::vox_workspace_bytes(n < 0 ? 0 : n, C, g.slab_tiles(),
                                    nisect < 0 ? 0 : nisect);
}

size_t gsv_voxelize_slab_workspace_bytes(int32_t n, int32_t C, int64_t nisect,
                                         const int32_t vol[3], int32_t tz0,
                                         int32_t tz1) {
    if (!vol || vol[0] <= 0 || vol[1] <= 0 || vol[2] <= 0) return 0;
    if (C < 1 || C > 4) return 0;
    const gsv::Geom g = gsv::make_geom(vol, tz0, tz1);
    if (g.tz0 < 0 || g.tz1 > g.Tz || g.tz0 > g.tz1) return 0;
    return gsv::vox_workspace_bytes(n < 0 ? 0 : n, C, g.slab_tiles(),
                                    nisect < 0 ? 0 : nisect);
}

int gsv_voxelize_forward(const int32_t vol[3], int32_t C, int32_t n,
                         int64_t nisect, const int32_t *ids,
                         const int32_t *bins, const float *pos,
                         const float *con, const float *inten, float *out,
                         void *ws, size_t ws_bytes, void *stream) {
    const char *fn = "gsv_voxelize_forward";
    if (!check_vol(vol, fn)) return GSV_ERR_INVALID_ARGUMENT;
    return forward_impl(fn, gsv::make_geom(vol), C, n, nisect, ids, bins, pos,
                        con, inten, out, ws, ws_bytes, stream);
}

int gsv_voxelize_forward_slab(const int32_t vol[3], int32_t tz0, int32_t tz1,
                              int32_t C, int32_t n, int64_t nisect,
                              const int32_t *ids, const int32_t *bins,
                              const float *pos, const float *con,
                              const float *inten, float *out, void *ws,
                              size_t ws_bytes, void *stream) {
    const char *fn = "gsv_voxelize_forward_slab";
    if (!check_vol(vol, fn)) return GSV_ERR_INVALID_ARGUMENT;
    return forward_impl(fn, gsv::make_geom(vol, tz0, tz1), C, n, nisect, ids,
                        bins, pos, con, inten, out, ws, ws_bytes, stream);
}

int gsv_voxelize_backward_per_gaussian(
    const int32_t vol[3], int32_t C, int32_t n, int64_t nisect,
    const int32_t *ids, const int32_t *bins, const float *pos,
    const float *con, const float *inten, const float *grad, float *pos_grad,
    float *con_grad, float *int_grad, void *ws, size_t ws_bytes,
    void *stream) {
    const char *fn = "gsv_voxelize_backward_per_gaussian";
    if (!check_vol(vol, fn)) return GSV_ERR_INVALID_ARGUMENT;
    return backward_impl(fn, true, gsv::make_geom(vol), C, n, nisect, ids,
                         bins, pos, con, inten, grad, pos_grad, con_grad,
                         int_grad, ws, ws_bytes, stream);
}

int gsv_voxelize_backward_per_gaussian_slab(
    const int32_t vol[3], int32_t tz0, int32_t tz1, int32_t C, int32_t n,
    int64_t nisect, const int32_t *ids, const int32_t *bins, const float *pos,
    const float *con, const float *inten, const float *grad, float *pos_grad,
    float *con_grad, float *int_grad, void *ws, size_t ws_bytes,
    void *stream) {
    const char *fn = "gsv_voxelize_backward_per_gaussian_slab";
    if (!check_vol(vol, fn)) return GSV_ERR_INVALID_ARGUMENT;
    return backward_impl(fn, true, gsv::make_geom(vol, tz0, tz1), C, n, nisect,
                         ids, bins, pos, con, inten, grad, pos_grad, con_grad,
                         int_grad, ws, ws_bytes, stream);
}

int gsv_voxelize_backward(const int32_t vol[3], int32_t C, int32_t n,
                          int64_t nisect, const int32_t *ids,
                          const int32_t *bins, const float *pos,
                          const float *con, const float *inten,
                          const float *grad, float *pos_grad, float *con_grad,
                          float *int_grad, void *ws, size_t ws_bytes,
                          void *stream) {
    const char *fn = "gsv_voxelize_backward";
    if (!check_vol(vol, fn)) return GSV_ERR_INVALID_ARGUMENT;
    return backward_impl(fn, false, gsv::make_geom(vol), C, n, nisect, ids,
                         bins, pos, con, inten, grad, pos_grad, con_grad,
                         int_grad, ws, ws_bytes, stream);
}

size_t gsv_l1_loss_workspace_bytes(int64_t n) {
    return gsv::l1_workspace_bytes(n < 0 ? 0 : n);
}

int gsv_l1_loss_forward(int64_t n, const float *vol, const float *target,
                        float denom, float *loss_out, void *ws,
                        size_t ws_bytes, void *stream) {
    const char *fn = "gsv_l1_loss_forward";
    GSV_REQUIRE(n >= 0 && loss_out && (n == 0 || (vol && target)),
                GSV_ERR_INVALID_ARGUMENT, "%s: bad arguments", fn);
    GSV_REQUIRE(denom != 0.f, GSV_ERR_INVALID_ARGUMENT, "%s: denom is 0", fn);
    const size_t need = gsv::l1_workspace_bytes(n);
    GSV_REQUIRE(ws && ws_bytes >= need, GSV_ERR_WORKSPACE_TOO_SMALL,
                "%s: workspace of %zu bytes given, %zu needed", fn, ws_bytes,
                need);
    return cuda_status(gsv::launch_sum(n, vol, target, 1.0 / (double)denom,
                                       loss_out, ws, as_stream(stream)),
                       fn);
}

int gsv_l1_loss_backward(int64_t n, const float *vol, const float *target,
                         const float *grad_loss, float denom, float *grad_vol,
                         void *stream) {
    const char *fn = "gsv_l1_loss_backward";
    GSV_REQUIRE(n >= 0 && (n == 0 || (vol && target && grad_loss && grad_vol)),
                GSV_ERR_INVALID_ARGUMENT, "%s: bad arguments", fn);
    GSV_REQUIRE(denom != 0.f, GSV_ERR_INVALID_ARGUMENT, "%s: denom is 0", fn);
    if (n == 0) return GSV_OK;
    return cuda_status(gsv::launch_l1_grad(n, vol, target, grad_loss,
                                           1.f / denom, grad_vol,
                                           as_stream(stream)),
                       fn);
}

size_t gsv_voxelize_l1_workspace_bytes(int32_t n, int32_t C, int64_t nisect,
                                       const int32_t vol[3], int32_t tz0,
                                       int32_t tz1) {
    if (!vol || vol[0] <= 0 || vol[1] <= 0 || vol[2] <= 0) return 0;
    if (C < 1 || C > 4) return 0;
    const gsv::Geom g = gsv::make_geom(vol, tz0, tz1);
    if (g.tz0 < 0 || g.tz1 > g.Tz || g.tz0 > g.tz1) return 0;
    const long long ni = nisect < 0 ? 0 : nisect;
    return l1_bin_part(g, ni, n < 0 ? 0 : n) +
           gsv::vox_workspace_bytes(n < 0 ? 0 : n, C, g.slab_tiles(), ni) +
           l1_tc_part(g, C, ni);
}

int gsv_voxelize_forward_l1(const int32_t vol[3], int32_t tz0, int32_t tz1,
                            int32_t C, int32_t n, int64_t nisect,
                            const int32_t *tile_min, const int32_t *tile_max,
                            const float *pos, const float *con,
                            const float *inten, const float *target,
                            float denom, int32_t *ids_out, int32_t *bins_out,
                            float *out, float *loss_out, int64_t *count_out,
                            float *overflow_out, void *ws, size_t ws_bytes,
                            void *stream) {
    const char *fn = "gsv_voxelize_forward_l1";
    if (!check_vol(vol, fn)) return GSV_ERR_INVALID_ARGUMENT;
    const gsv::Geom g = gsv::make_geom(vol, tz0, tz1);
    if (!check_slab(g, fn)) return GSV_ERR_INVALID_ARGUMENT;
    GSV_REQUIRE(C >= 1 && C <= 4, GSV_ERR_UNSUPPORTED_CHANNELS,
                "%s: %d channels requested, 1..4 supported", fn, C);
    GSV_REQUIRE(n >= 0 && nisect >= 0, GSV_ERR_INVALID_ARGUMENT,
                "%s: negative size", fn);
    GSV_REQUIRE(nisect <= INT32_MAX && g.slab_tiles() <= INT32_MAX,
                GSV_ERR_SIZE_OVERFLOW, "%s: sizes exceed int32", fn);
    const size_t need = gsv_voxelize_l1_workspace_bytes(n, C, nisect, vol,
                                                        tz0, tz1);
    GSV_REQUIRE(ws && ws_bytes >= need, GSV_ERR_WORKSPACE_TOO_SMALL,
                "%s: workspace of %zu bytes given, %zu needed", fn, ws_bytes,
                need);
    const long long nvox =
        (long long)(g.z_end() - g.z_begin()) * g.Y * g.X * C;
    GSV_REQUIRE((out && target) || nvox == 0, GSV_ERR_INVALID_ARGUMENT,
                "%s: out_vol or target is null", fn);
    GSV_REQUIRE(loss_out && denom != 0.f, GSV_ERR_INVALID_ARGUMENT,
                "%s: loss_out is null or denom is 0", fn);
    GSV_REQUIRE(g.slab_tiles() == 0 || bins_out, GSV_ERR_INVALID_ARGUMENT,
                "%s: tile_bins is null", fn);
    GSV_REQUIRE(nisect == 0 || (ids_out && tile_min && tile_max && pos && con &&
                                inten),
                GSV_ERR_INVALID_ARGUMENT, "%s: null input pointer", fn);
    cudaStream_t s = as_stream(stream);
    char *bin_ws = static_cast<char *>(ws);
    char *vox_ws = bin_ws + l1_bin_part(g, nisect, n);
    gsv::enable_large_smem();
    // the binning also scans and writes the backward's work plan
    const gsv::ItemScan items =
        gsv::vox_item_scan(vox_ws, n, C, g.slab_tiles(), nisect);
    cudaError_t err = gsv::launch_binning(
        n, nisect, tile_min, tile_max, g.Tx, g.Ty, g.tz0, g.tz1, ids_out,
        bins_out, bin_ws, s, reinterpret_cast<long long *>(count_out),
        overflow_out, &items);
    if (err) return cuda_status(err, fn);
    if (nisect == 0) {
        // empty volume: loss = sum |target| / denom
        err = cudaMemsetAsync(out, 0, sizeof(float) * nvox, s);
        if (err) return cuda_status(err, fn);
        return cuda_status(gsv::launch_empty_l1(nvox, target,
                                                1.0 / (double)denom, loss_out,
                                                vox_ws, s),
                           fn);
    }
    // tensor-core backward selected: also its inputs
    TcBuffers tcb = {nullptr, nullptr};
    if (use_tc(C)) tcb = l1_tc_buffers(ws, g, C, n, nisect);
    err = gsv::launch_vox_forward_ex(g, C, n, nisect, ids_out, bins_out, pos,
                                     con, inten, out, vox_ws, s, target,
                                     loss_out, 1.0 / (double)denom,
                                     tcb.sign_plane, tcb.tile_of);
    return cuda_status(err, fn);
}

int gsv_voxelize_backward_per_gaussian_l1(
    const int32_t vol[3], int32_t tz0, int32_t tz1, int32_t C, int32_t n,
    int64_t nisect, const int32_t *ids, const int32_t *bins, const float *pos,
    const float *con, const float *inten, const float *out_vol,
    const float *target, const float *grad_loss, float denom, float *pos_grad,
    float *con_grad, float *int_grad, void *ws, size_t ws_bytes,
    void *stream) {
    const char *fn = "gsv_voxelize_backward_per_gaussian_l1";
    if (!check_vol(vol, fn)) return GSV_ERR_INVALID_ARGUMENT;
    const gsv::Geom g = gsv::make_geom(vol, tz0, tz1);
    if (!check_slab(g, fn)) return GSV_ERR_INVALID_ARGUMENT;
    GSV_REQUIRE(C >= 1 && C <= 4, GSV_ERR_UNSUPPORTED_CHANNELS,
                "%s: %d channels requested, 1..4 supported", fn, C);
    GSV_REQUIRE(n >= 0 && nisect >= 0 && nisect <= INT32_MAX,
                GSV_ERR_INVALID_ARGUMENT, "%s: bad sizes", fn);
    const size_t need = gsv_voxelize_l1_workspace_bytes(n, C, nisect, vol,
                                                        tz0, tz1);
    GSV_REQUIRE(ws && ws_bytes >= need, GSV_ERR_WORKSPACE_TOO_SMALL,
                "%s: workspace of %zu bytes given, %zu needed", fn, ws_bytes,
                need);
    GSV_REQUIRE(n == 0 || (pos_grad && con_grad && int_grad),
                GSV_ERR_INVALID_ARGUMENT, "%s: null gradient output", fn);
    GSV_REQUIRE(nisect == 0 || (ids && bins && pos && con && inten && out_vol &&
                                target && grad_loss),
                GSV_ERR_INVALID_ARGUMENT, "%s: null input pointer", fn);
    GSV_REQUIRE(denom != 0.f, GSV_ERR_INVALID_ARGUMENT, "%s: denom is 0", fn);
    char *vox_ws = static_cast<char *>(ws) + l1_bin_part(g, nisect, n);
    gsv::TcInputs tc;
    const gsv::TcInputs *tcp = nullptr;
    if (use_tc(C)) {
        const TcBuffers b = l1_tc_buffers(ws, g, C, n, nisect);
        tc.sign_plane = b.sign_plane;
        tc.tile_of = b.tile_of;
        tc.pair_total = gsv::bin_pair_total(ws, g.slab_tiles());
        tcp = &tc;
    }
    return cuda_status(gsv::launch_vox_backward_gauss(
                           g, C, n, nisect, ids, bins, pos, con, inten,
                           out_vol, pos_grad, con_grad, int_grad, vox_ws,
                           as_stream(stream), target, grad_loss, 1.f / denom,
                           gsv::kBwdPrepared, tcp),
                       fn);
}

int gsv_set_tensor_core_backward(int32_t enable) {
    const int prev = g_use_tc_backward ? 1 : 0;
    g_use_tc_backward = enable != 0;
    return prev;
}

int gsv_device_error(int32_t *flag_out, int32_t clear) {
    const char *fn = "gsv_device_error";
    GSV_REQUIRE(flag_out, GSV_ERR_INVALID_ARGUMENT, "%s: flag_out is null", fn);
    const int a = gsv::tc_error_flag(clear != 0);
    const int b = gsv::peer_error_flag(clear != 0);
    GSV_REQUIRE(a >= 0 && b >= 0, GSV_ERR_CUDA, "%s: could not read the device flags",
                fn);
    *flag_out = (a ? 1 : 0) | (b ? 2 : 0);
    return GSV_OK;
}

size_t gsv_halo_workspace_bytes(int32_t n, int32_t world) {
    if (n < 0 || world < 1 || world > gsv::kHaloMaxRanks) return 0;
    return gsv::halo_workspace_bytes(n, world);
}

static int halo_pack_impl(const char *fn, int32_t n, int32_t C,
                          const float *pos3d_radii, const float *conics,
                          const float *intensities, const int32_t *tile_min,
                          const int32_t *tile_max, int32_t world, int32_t rank,
                          const int32_t *slab_tz, const int64_t *seg_off,
                          const int32_t *seg_slots, float *send,
                          const int64_t *seg_dst, int32_t *slot_map,
                          int64_t *counts_out, void *ws, size_t ws_bytes,
                          void *stream) {
    gsv::HaloPeers P;
    long long total;
    GSV_REQUIRE(n >= 0 && C >= 1 && C <= 4 && slab_tz &&
                    make_peers(world, rank, slab_tz, seg_off, seg_slots, P, total),
                GSV_ERR_INVALID_ARGUMENT, "%s: bad sizes or peer description", fn);
    GSV_REQUIRE(ws && ws_bytes >= gsv::halo_workspace_bytes(n, world),
                GSV_ERR_WORKSPACE_TOO_SMALL, "%s: workspace too small", fn);
    GSV_REQUIRE(slot_map && (n == 0 || (pos3d_radii && conics && intensities &&
                                        tile_min && tile_max)),
                GSV_ERR_INVALID_ARGUMENT, "%s: null pointer", fn);
    GSV_REQUIRE(set_destinations(P, send, seg_dst, gsv::kHaloRec),
                GSV_ERR_INVALID_ARGUMENT,
                "%s: missing or misaligned segment destination", fn);
    return cuda_status(gsv::launch_halo_pack(n, C, pos3d_radii, conics,
                                             intensities, tile_min, tile_max,
                                             P, slot_map,
                                             reinterpret_cast<long long *>(counts_out),
                                             ws, as_stream(stream)),
                       fn);
}

int gsv_halo_pack(int32_t n, int32_t C, const float *pos3d_radii,
                  const float *conics, const float *intensities,
                  const int32_t *tile_min, const int32_t *tile_max,
                  int32_t world, int32_t rank, const int32_t *slab_tz,
                  const int64_t *seg_off, const int32_t *seg_slots,
                  float *send, int32_t *slot_map, int64_t *counts_out,
                  void *ws, size_t ws_bytes, void *stream) {
    return halo_pack_impl("gsv_halo_pack", n, C, pos3d_radii, conics,
                          intensities, tile_min, tile_max, world, rank, slab_tz,
                          seg_off, seg_slots, send, nullptr, slot_map,
                          counts_out, ws, ws_bytes, stream);
}

int gsv_halo_pack_peers(int32_t n, int32_t C, const float *pos3d_radii,
                        const float *conics, const float *intensities,
                        const int32_t *tile_min, const int32_t *tile_max,
                        int32_t world, int32_t rank, const int32_t *slab_tz,
                        const int64_t *seg_off, const int32_t *seg_slots,
                        const int64_t *seg_dst, int32_t *slot_map,
                        int64_t *counts_out, void *ws, size_t ws_bytes,
                        void *stream) {
    return halo_pack_impl("gsv_halo_pack_peers", n, C, pos3d_radii, conics,
                          intensities, tile_min, tile_max, world, rank, slab_tz,
                          seg_off, seg_slots, nullptr, seg_dst, slot_map,
                          counts_out, ws, ws_bytes, stream);
}

int gsv_halo_unpack(int32_t n_own, int32_t C, int32_t world,
                            int32_t rank, const int64_t *seg_off,
                            const int32_t *seg_slots, const float *recv,
                            float *pos3d_radii, float *conics,
                            float *intensities, int32_t *tile_min,
                            int32_t *tile_max, float *flags, void *stream) {
    const char *fn = "gsv_halo_unpack";
    gsv::HaloPeers R;
    long long total;
    GSV_REQUIRE(n_own >= 0 && C >= 1 && C <= 4 &&
                    make_peers(world, rank, nullptr, seg_off, seg_slots, R, total),
                GSV_ERR_INVALID_ARGUMENT, "%s: bad sizes or peer description", fn);
    GSV_REQUIRE(total == 0 || (recv && pos3d_radii && conics && intensities &&
                               tile_min && tile_max && flags),
                GSV_ERR_INVALID_ARGUMENT, "%s: null pointer", fn);
    // the peers' headers (overflow bits) are read whenever there are peers
    GSV_REQUIRE(world == 1 || (recv && flags), GSV_ERR_INVALID_ARGUMENT,
                "%s: null pointer", fn);
    return cuda_status(gsv::launch_halo_unpack(n_own, C, R, total, recv,
                                               pos3d_radii, conics, intensities,
                                               tile_min, tile_max, flags,
                                               as_stream(stream)),
                       fn);
}

static int halo_pack_grads_impl(const char *fn, int32_t n_own, int32_t C,
                                int32_t world, int32_t rank,
                                const int64_t *seg_off, const int32_t *seg_slots,
                                const float *pos3d_radii_grad,
                                const float *conics_grad,
                                const float *intensities_grad, const float *loss,
                                const float *flags, float *send,
                                const int64_t *seg_dst, void *stream) {
    gsv::HaloPeers R;
    long long total;
    GSV_REQUIRE(n_own >= 0 && C >= 1 && C <= 4 &&
                    make_peers(world, rank, nullptr, seg_off, seg_slots, R, total),
                GSV_ERR_INVALID_ARGUMENT, "%s: bad sizes or peer description", fn);
    GSV_REQUIRE(loss && flags &&
                    (total == 0 || (pos3d_radii_grad && conics_grad &&
                                    intensities_grad)),
                GSV_ERR_INVALID_ARGUMENT, "%s: null pointer", fn);
    GSV_REQUIRE(set_destinations(R, send, seg_dst, gsv::kHaloGrad),
                GSV_ERR_INVALID_ARGUMENT,
                "%s: missing or misaligned segment destination", fn);
    return cuda_status(gsv::launch_halo_pack_grads(
                           n_own, C, R, total, pos3d_radii_grad, conics_grad,
                           intensities_grad, loss, flags, as_stream(stream)),
                       fn);
}

int gsv_halo_pack_grads(int32_t n_own, int32_t C, int32_t world, int32_t rank,
                        const int64_t *seg_off, const int32_t *seg_slots,
                        const float *pos3d_radii_grad, const float *conics_grad,
                        const float *intensities_grad, const float *loss,
                        const float *flags, float *send, void *stream) {
    return halo_pack_grads_impl("gsv_halo_pack_grads", n_own, C, world, rank,
                                seg_off, seg_slots, pos3d_radii_grad,
                                conics_grad, intensities_grad, loss, flags, send,
                                nullptr, stream);
}

int gsv_halo_pack_grads_peers(int32_t n_own, int32_t C, int32_t world,
                              int32_t rank, const int64_t *seg_off,
                              const int32_t *seg_slots,
                              const float *pos3d_radii_grad,
                              const float *conics_grad,
                              const float *intensities_grad, const float *loss,
                              const float *flags, const int64_t *seg_dst,
                              void *stream) {
    return halo_pack_grads_impl("gsv_halo_pack_grads_peers", n_own, C, world,
                                rank, seg_off, seg_slots, pos3d_radii_grad,
                                conics_grad, intensities_grad, loss, flags,
                                nullptr, seg_dst, stream);
}

int gsv_halo_accumulate(int32_t n, int32_t C, int32_t world,
                                int32_t rank, const int64_t *seg_off,
                                const int32_t *slot_map, const float *recv,
                                float *pos3d_radii_grad, float *conics_grad,
                                float *intensities_grad, const float *loss,
                                const float *flags, float *out, void *stream) {
    const char *fn = "gsv_halo_accumulate";
    gsv::HaloPeers P;
    long long total;
    int32_t dummy_slots[gsv::kHaloMaxRanks] = {0};
    GSV_REQUIRE(n >= 0 && C >= 1 && C <= 4 &&
                    make_peers(world, rank, nullptr, seg_off, dummy_slots, P, total),
                GSV_ERR_INVALID_ARGUMENT, "%s: bad sizes or peer description", fn);
    GSV_REQUIRE(recv && loss && flags && out &&
                    (n == 0 || (slot_map && pos3d_radii_grad && conics_grad &&
                                intensities_grad)),
                GSV_ERR_INVALID_ARGUMENT, "%s: null pointer", fn);
    return cuda_status(gsv::launch_halo_accumulate(
                           n, C, P, slot_map, recv, pos3d_radii_grad,
                           conics_grad, intensities_grad, loss, flags, out,
                           as_stream(stream)),
                       fn);
}

}  // extern "C"

// ------------------------------------------------------------ SSIM and TV

namespace {

// 0 if the planar volume description is valid, else the status (message set)
int check_dhw(int32_t nch, const int32_t *dhw, const char *fn) {
    if (nch < 1 || !dhw || dhw[0] <= 0 || dhw[1] <= 0 || dhw[2] <= 0)
        return fail(GSV_ERR_INVALID_ARGUMENT, "%s: bad channel count or volume size", fn);
    if ((long long)nch * dhw[0] * dhw[1] * dhw[2] > (1LL << 40))
        return fail(GSV_ERR_SIZE_OVERFLOW, "%s: volume too large", fn);
    if ((dhw[0] + 31) / 32 * (long long)nch > 65535)
        return fail(GSV_ERR_SIZE_OVERFLOW, "%s: too many channels x z-runs", fn);
    return GSV_OK;
}

const gsv::SsWindowHost &ssim_window_15() {
    static const gsv::SsWindowHost w = gsv::ssim_window(1.5);
    return w;
}

}  // namespace

extern "C" {

size_t gsv_ssim3d_workspace_bytes(int32_t channels, const int32_t dhw[3]) {
    if (channels < 1 || !dhw || dhw[0] <= 0 || dhw[1] <= 0 || dhw[2] <= 0) return 0;
    return gsv::ssim_workspace_bytes(channels, dhw[0], dhw[1], dhw[2]);
}

int gsv_ssim3d_forward(int32_t channels, const int32_t dhw[3], const float *img1,
                       const float *img2, float c1, float c2, float *ssim_out,
                       void *ws, size_t ws_bytes, void *stream) {
    const char *fn = "gsv_ssim3d_forward";
    if (const int st = check_dhw(channels, dhw, fn)) return st;
    const size_t need = gsv_ssim3d_workspace_bytes(channels, dhw);
    GSV_REQUIRE(ws && ws_bytes >= need, GSV_ERR_WORKSPACE_TOO_SMALL,
                "%s: workspace of %zu bytes given, %zu needed", fn, ws_bytes, need);
    GSV_REQUIRE(img1 && img2 && ssim_out, GSV_ERR_INVALID_ARGUMENT,
                "%s: null pointer", fn);
    return cuda_status(gsv::launch_ssim_forward(channels, dhw[0], dhw[1], dhw[2],
                                                img1, img2, c1, c2, ssim_window_15(),
                                                ssim_out, ws, as_stream(stream)),
                       fn);
}

int gsv_ssim3d_backward(int32_t channels, const int32_t dhw[3], const float *img1,
                        const float *img2, const float *grad_out, const void *ws,
                        size_t ws_bytes, float *grad_img1, void *stream) {
    const char *fn = "gsv_ssim3d_backward";
    if (const int st = check_dhw(channels, dhw, fn)) return st;
    const size_t need = gsv_ssim3d_workspace_bytes(channels, dhw);
    GSV_REQUIRE(ws && ws_bytes >= need, GSV_ERR_WORKSPACE_TOO_SMALL,
                "%s: workspace of %zu bytes given, %zu needed", fn, ws_bytes, need);
    GSV_REQUIRE(img1 && img2 && grad_out && grad_img1, GSV_ERR_INVALID_ARGUMENT,
                "%s: null pointer", fn);
    return cuda_status(gsv::launch_ssim_backward(channels, dhw[0], dhw[1], dhw[2],
                                                 img1, img2, ssim_window_15(),
                                                 grad_out, ws, grad_img1,
                                                 as_stream(stream)),
                       fn);
}

size_t gsv_tv3d_workspace_bytes(int32_t channels, const int32_t dhw[3]) {
    if (channels < 1 || !dhw || dhw[0] <= 0 || dhw[1] <= 0 || dhw[2] <= 0) return 0;
    return gsv::tv_workspace_bytes(channels, dhw[0], dhw[1], dhw[2]);
}

int gsv_tv3d(int32_t channels, const int32_t dhw[3], const float *vol,
             int32_t isotropic, float eps, float *value_out, const float *grad_out,
             float *grad_vol, void *ws, size_t ws_bytes, void *stream) {
    const char *fn = "gsv_tv3d";
    if (const int st = check_dhw(channels, dhw, fn)) return st;
    const size_t need = gsv_tv3d_workspace_bytes(channels, dhw);
    GSV_REQUIRE(ws && ws_bytes >= need, GSV_ERR_WORKSPACE_TOO_SMALL,
                "%s: workspace of %zu bytes given, %zu needed", fn, ws_bytes, need);
    GSV_REQUIRE(vol && (value_out || grad_vol), GSV_ERR_INVALID_ARGUMENT,
                "%s: null pointer", fn);
    GSV_REQUIRE(!grad_vol || grad_out, GSV_ERR_INVALID_ARGUMENT,
                "%s: grad_vol needs grad_out", fn);
    GSV_REQUIRE(!isotropic || eps > 0.f, GSV_ERR_INVALID_ARGUMENT,
                "%s: isotropic TV needs eps > 0", fn);
    return cuda_status(gsv::launch_tv(channels, dhw[0], dhw[1], dhw[2], vol,
                                      isotropic, eps, value_out, grad_out, grad_vol,
                                      ws, as_stream(stream)),
                       fn);
}

}  // extern "C"

extern "C" int gsv_peer_barrier(int32_t world, int32_t rank, const int64_t *sig_ptrs,
                                int32_t *epoch, void *stream) {
    const char *fn = "gsv_peer_barrier";
    GSV_REQUIRE(world >= 1 && world <= gsv::kHaloMaxRanks && rank >= 0 &&
                    rank < world && sig_ptrs && epoch,
                GSV_ERR_INVALID_ARGUMENT, "%s: bad ranks or null pointer", fn);
    for (int d = 0; d < world; ++d)
        GSV_REQUIRE(sig_ptrs[d] != 0 && (sig_ptrs[d] & 3) == 0,
                    GSV_ERR_INVALID_ARGUMENT, "%s: bad signal address of rank %d",
                    fn, d);
    return cuda_status(gsv::launch_peer_barrier(
                           world, rank, reinterpret_cast<const long long *>(sig_ptrs),
                           epoch, as_stream(stream)),
                       fn);
}
