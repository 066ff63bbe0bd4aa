// context.cu -- the nerf.h C ABI and the additive nerf_b200.h exports.
//
// A context owns, on the device that is current at creation:
//   scene arena     images (RGBA8), cameras, the nerf_inference image
//   model arena     flat parameters (fp32 masters, fp16 mirror, Adam m/v),
//                   fp16 hash-table gradients, fp32 MLP gradients (+ loss
//                   slot), the device step state
//   occupancy arena density grid (padded to whole 32-cell words), bitfield
//   batch arena     (sized at nerf_configure_training) per-ray counts,
//                   chunk starts and kept-step lists, compacted rays and samples, hash
//                   features, raw field outputs and their gradients, the
//                   backward kernel's weight-gradient partials, the
//                   occupancy query window
// The training step is one CUDA graph captured at configure time: occupancy
// query -> occupancy update -> sampler (bitfield tests, scan, sample writes)
// -> field forward -> composite + loss -> MLP backward -> hash-table scatter
// -> [data parallel: weight-gradient reduce, then the gradient exchange --
// peer mode: barrier, owned-range reduce over NVLink, barrier; or an NCCL
// all-reduce] -> gradient statistics / step commit -> the next step's march
// -> Adam [peer mode: writing every rank's mirror, then a barrier].  Every
// kernel reads the step number and
// the batch sizes from device memory, so nerf_train_step is one
// cudaGraphLaunch (reference backend-cuda.cu:2405-2420).
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/nerf.h"
#include "../../include/nerf_b200.h"
#include "kernels.h"

namespace nb {
namespace {

static_assert(sizeof(NerfB200GridLayout) == sizeof(GridLayout), "grid layout mirror");
static_assert(sizeof(NerfB200RayRecord) == sizeof(RayRecord), "ray record mirror");
static_assert(sizeof(StatsBlock) == sizeof(NerfTrainStats), "stats mirror");

constexpr uint32_t kMaxStepsPerRay = 4096;  // the reference allows 256
constexpr int kStepKernels = 14;            // timed segments of one training step
// Exported peer handle: the model arena's CUDA IPC handle, then the arena's
// size and parameter count (all ranks' must agree), then a format word.
constexpr uint32_t kDpHandleBytes = NERF_B200_DP_HANDLE_BYTES;
constexpr uint32_t kDpHandleMagic = 0x4E42504Bu;

// ---------------------------------------------------------------- helpers
uint64_t align_up(uint64_t v, uint64_t a) { return (v + a - 1u) / a * a; }

struct Arena {
    unsigned char* base = nullptr;
    uint64_t size = 0;
    uint64_t align = 256;
    uint64_t add(uint64_t bytes) {
        size = align_up(size, align);
        const uint64_t off = size;
        size += std::max<uint64_t>(bytes, 1u);
        return off;
    }
    cudaError_t alloc() {
        release();
        if (size == 0u) return cudaSuccess;
        return cudaMalloc(&base, size);
    }
    void release() {
        if (base) cudaFree(base);
        base = nullptr;
    }
    template <class T>
    T* at(uint64_t off) const {
        return reinterpret_cast<T*>(base + off);
    }
};

// Hash-grid layout rule (the CPU oracle restates it independently):
// b = (N_max/N_min)^(1/(L-1)); s_l = float(N_min * b^l - 1) in double;
// R_l = ceil(s_l) + 2 vertices per axis; dense when R_l^3 <= T; level sizes
// R_l^3 rounded up to 8 (dense) or T (hashed), stored back to back.
int grid_layout(uint32_t L, uint32_t log2T, uint32_t base, uint32_t maxres, GridLayout* g) {
    if (L == 0u || L > kMaxLevels || log2T < 4u || log2T > 26u || base < 2u || maxres < base) return 1;
    std::memset(g, 0, sizeof(*g));
    g->n_levels = L;
    g->log2_hashmap_size = log2T;
    g->base_resolution = base;
    g->max_resolution = maxres;
    const double step = L > 1u ? std::log2(static_cast<double>(maxres) / base) / static_cast<double>(L - 1u) : 0.0;
    const uint64_t T = 1ull << log2T;
    uint64_t off = 0;
    for (uint32_t l = 0; l < L; ++l) {
        const float s = static_cast<float>(std::exp2(l * step) * static_cast<double>(base) - 1.0);
        const uint32_t R = static_cast<uint32_t>(std::ceil(static_cast<double>(s))) + 2u;
        const uint64_t cells = static_cast<uint64_t>(R) * R * R;
        const bool dense = cells <= T;
        g->scale[l] = s;
        g->resolution[l] = R;
        g->dense[l] = dense ? 1u : 0u;
        g->offset[l] = static_cast<uint32_t>(off);
        off += dense ? align_up(cells, 8u) : T;
        if (off >= (1ull << 31)) return 2;
    }
    g->offset[L] = static_cast<uint32_t>(off);
    return 0;
}

// splitmix64 stream of the reference weight init (backend-cuda.cu:1810-1847).
struct SplitMix {
    uint64_t state;
    SplitMix(uint64_t a, uint64_t b) : state((a + 0x9e3779b97f4a7c15ull) ^ (b * 0xbf58476d1ce4e5b9ull)) {}
    float unit() {  // [-1, 1) from 24 bits
        state += 0x9e3779b97f4a7c15ull;
        uint64_t z = state;
        z = (z ^ (z >> 30u)) * 0xbf58476d1ce4e5b9ull;
        z = (z ^ (z >> 27u)) * 0x94d049bb133111ebull;
        z ^= z >> 31u;
        return static_cast<float>(static_cast<uint32_t>(z >> 32u) >> 8u) * (1.0f / 16777216.0f) * 2.0f - 1.0f;
    }
};
void xavier(SplitMix& rng, uint32_t fan_in, uint32_t fan_out, float* out) {
    const float scale = std::sqrt(6.0f / static_cast<float>(fan_in + fan_out));
    for (uint64_t i = 0; i < static_cast<uint64_t>(fan_in) * fan_out; ++i) out[i] = rng.unit() * scale;
}

float env_float(const char* name, float dflt) {
    const char* v = std::getenv(name);
    return (v && *v) ? static_cast<float>(std::atof(v)) : dflt;
}
uint32_t env_u32(const char* name, uint32_t dflt) {
    const char* v = std::getenv(name);
    return (v && *v) ? static_cast<uint32_t>(std::strtoul(v, nullptr, 10)) : dflt;
}

NerfStatus cuda_status(cudaError_t e) { return e == cudaSuccess ? NERF_STATUS_OK : NERF_STATUS_CUDA_ERROR; }
#define NB_TRY(expr)                                           \
    do {                                                       \
        const cudaError_t e_ = (expr);                         \
        if (e_ != cudaSuccess) return NERF_STATUS_CUDA_ERROR;  \
    } while (0)

// Kernel attributes are set once per device.
std::mutex g_attr_mu;
bool g_attr_done[64] = {};

// ------------------------------------------------------ NCCL (loaded lazily)
struct Nccl {
    bool loaded = false;
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) comm_init_rank = nullptr;
    decltype(&ncclAllReduce) all_reduce = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclCommDestroy) comm_destroy = nullptr;
    bool load() {
        if (loaded) return true;
        // In a process that already loaded NCCL (e.g. through PyTorch) this
        // returns that library instead of loading a second one.
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return false;
        get_unique_id = reinterpret_cast<decltype(get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
        comm_init_rank = reinterpret_cast<decltype(comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
        all_reduce = reinterpret_cast<decltype(all_reduce)>(dlsym(h, "ncclAllReduce"));
        all_gather = reinterpret_cast<decltype(all_gather)>(dlsym(h, "ncclAllGather"));
        comm_destroy = reinterpret_cast<decltype(comm_destroy)>(dlsym(h, "ncclCommDestroy"));
        loaded = get_unique_id && comm_init_rank && all_reduce && all_gather && comm_destroy;
        return loaded;
    }
};
Nccl g_nccl;
std::mutex g_nccl_mu;

}  // namespace

cudaError_t ensure_attributes() {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lk(g_attr_mu);
    if (dev >= 0 && dev < 64 && g_attr_done[dev]) return cudaSuccess;
    e = field_init_attributes();
    if (e == cudaSuccess && dev >= 0 && dev < 64) g_attr_done[dev] = true;
    return e;
}

// ------------------------------------------------------------------ context
struct Context {
    std::mutex mu;
    int device = 0;
    cudaStream_t stream = nullptr;
    NerfB200Options opt{};
    GridLayout grid{};
    LevelTable lt{};
    uint64_t n_grid = 0, n_params = 0;
    // scene
    uint32_t n_images = 0, width = 0, height = 0;
    float fx = 0, fy = 0, cx = 0, cy = 0;
    uint32_t grid_res = 0, cell_count = 0, words = 0;
    uint32_t max_sample_steps = 0, max_batch_rays = 0;
    uint64_t alignment = 256;
    Arena scene, model, occ, batch, render;
    uint8_t* images = nullptr;
    float* cams = nullptr;
    uint32_t* inference_rgba = nullptr;
    float* master = nullptr;
    __half* p16 = nullptr;
    float* m = nullptr;
    float* v = nullptr;
    __half* grid_grad = nullptr;
    float* mlp_grad = nullptr;
    DeviceState* state = nullptr;
    // Mapped pinned mirror of the step statistics, written by the statistics
    // kernel; current while the last writer of the device statistics was a
    // step (host writes of the device state make it stale).
    StatsBlock* stats_host = nullptr;
    StatsBlock* stats_host_dev = nullptr;
    bool stats_host_current = false;
    float* density = nullptr;
    uint32_t* bitfield = nullptr;
    uint32_t* full_bitfield = nullptr;  // all cells occupied (render before any occupancy exists)
    bool occupancy_valid = false;
    // batch
    uint32_t* ray_counts = nullptr;
    float* kept_t = nullptr;
    float* chunk_t = nullptr;
    RayGeom* geom = nullptr;
    uint32_t* ray_offset = nullptr;
    uint32_t* ray_slot = nullptr;
    RayRecord* rays = nullptr;
    uint32_t* ray_index = nullptr;
    float4* pos_dt = nullptr;
    uint32_t* sample_ray = nullptr;
    void* feat = nullptr;
    float4* raw = nullptr;
    float4* dout = nullptr;
    void* dfeat = nullptr;  // feature gradients of the training backward (fp16 x 32 per sample)
    float* partials = nullptr;
    float* occ_sigma = nullptr;
    uint32_t n_partials = 0, fwd_blocks = 0;
    bool mlp_tc = false;  // training backward MLP on tcgen05 (NERF_B200_MLP_TC)
    // render
    uint32_t* render_rgba = nullptr;
    uint32_t* render_counter = nullptr;
    unsigned long long* render_samples = nullptr;
    uint32_t render_w = 0, render_h = 0;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    // training
    bool configured = false;
    NerfTrainingConfig cfg{};
    TrainConsts tc{};
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    uint32_t host_generation = 0;
    // data parallel
    ncclComm_t comm = nullptr;
    uint32_t dp_rank = 0, dp_world = 1;
    // Peer mode: every rank's model arena mapped here (own base at dp_rank).
    bool dp_peer = false;
    unsigned char* peer_model[kMaxDpWorld] = {};
    float* dp_gsum = nullptr;   // owned range of summed gradients
    DpSync* dp_sync = nullptr;  // this rank's synchronisation words (model arena)
    // Wait limit of the barriers (NERF_B200_DP_TIMEOUT_MS, default 5 s); dp_watch:
    // nerf_read_train_stats reports a barrier that ran out (peer mode, or after
    // nerf_b200_dp_barrier_test); dp_absent: the never-written rank of that test.
    uint64_t dp_timeout_ns = 5000000000ull;
    bool dp_watch = false;
    DpSync* dp_absent = nullptr;
    float* mlp_sum = nullptr;   // MLP gradients + loss summed over the ranks (model arena)
    DpPeers dp_peers() const;
    uint64_t dp_lo(uint32_t r) const { return (n_grid / 8u) * r / dp_world * 8u; }
    template <class T>
    T* peer(uint32_t r, const T* local) const {  // the same buffer in rank r's model arena
        return reinterpret_cast<T*>(peer_model[r] + (reinterpret_cast<const unsigned char*>(local) - model.base));
    }
    NerfStatus open_peers();
    // Maps the other ranks' model arenas from their exported handles (world x
    // kDpHandleBytes); false when any cannot be opened (nothing stays mapped).
    bool map_peers(const unsigned char* handles);
    bool dp_active() const { return dp_world > 1u && (comm != nullptr || dp_peer); }
    // Host copy of a buffer of the model arena whose grid part is sharded over
    // the ranks in peer mode (masters, moments): each range from its owner.
    cudaError_t read_sharded(void* host, const float* local, uint64_t n) const;

    ~Context() { release_all(); }
    void release_graph() {
        if (exec) cudaGraphExecDestroy(exec);
        if (graph) cudaGraphDestroy(graph);
        exec = nullptr;
        graph = nullptr;
    }
    void release_all() {
        if (stream) cudaStreamSynchronize(stream);
        release_graph();
        scene.release();
        model.release();
        occ.release();
        batch.release();
        render.release();
        if (ev0) cudaEventDestroy(ev0);
        if (ev1) cudaEventDestroy(ev1);
        ev0 = ev1 = nullptr;
        for (uint32_t r = 0; r < kMaxDpWorld; ++r)
            if (peer_model[r] && r != dp_rank) cudaIpcCloseMemHandle(peer_model[r]);
        for (auto& p : peer_model) p = nullptr;
        dp_peer = false;
        if (comm && g_nccl.loaded) g_nccl.comm_destroy(comm);
        comm = nullptr;
        if (dp_absent) cudaFree(dp_absent);
        dp_absent = nullptr;
        if (stream) cudaStreamDestroy(stream);
        stream = nullptr;
        if (stats_host) cudaFreeHost(stats_host);
        stats_host = stats_host_dev = nullptr;
        stats_host_current = false;
    }
    NerfStatus init(const NerfCreateDesc& d, const NerfB200Options& o);
    NerfStatus configure(const NerfTrainingConfig& c);
    NerfStatus capture_graph();
    cudaError_t enqueue_step(cudaStream_t s, cudaEvent_t* ev);
    NerfStatus ensure_render_buffers(uint32_t w, uint32_t h);
    NerfStatus render_view(const float* c2w, uint32_t w, uint32_t h, float fx_, float fy_, float cx_, float cy_,
                           uint32_t max_steps, float stop, uint32_t tile, uint32_t rank, uint32_t world,
                           NerfB200RenderInfo* info);
    FieldArgs field_args() const;
    SamplerArgs sampler_args() const;
    void fill_aabb(float* mn, float* mx, float* size, const NerfTrainingConfig* with = nullptr) const;
    void base_aabb(float* mn, float* mx, const NerfTrainingConfig* with = nullptr) const;
    CascadeBox cascade_box(const NerfTrainingConfig* with = nullptr) const;
};

FieldArgs Context::field_args() const {
    FieldArgs a{};
    a.lt = lt;
    a.params16 = p16;
    a.mlp_offset = static_cast<uint32_t>(n_grid);
    a.state = state;
    fill_aabb(a.aabb_min, a.aabb_max, a.aabb_size);
    a.casc = cascade_box();
    return a;
}

// The configured AABB (cascade 0), or [0,1]^3 before configuration (the
// reference renders that box then).  During configure the new configuration
// is passed explicitly.
void Context::base_aabb(float* mn, float* mx, const NerfTrainingConfig* with) const {
    const NerfTrainingConfig* c = with ? with : (configured ? &cfg : nullptr);
    if (c) {
        mn[0] = c->aabb_min_x;
        mn[1] = c->aabb_min_y;
        mn[2] = c->aabb_min_z;
        mx[0] = c->aabb_max_x;
        mx[1] = c->aabb_max_y;
        mx[2] = c->aabb_max_z;
    } else {
        mn[0] = mn[1] = mn[2] = 0.0f;
        mx[0] = mx[1] = mx[2] = 1.0f;
    }
}

// Cascade k covers centre +- half * 2^k, centre = (min + max) / 2,
// half = size / 2 (exact).
CascadeBox Context::cascade_box(const NerfTrainingConfig* with) const {
    CascadeBox b{};
    float mn[3], mx[3];
    base_aabb(mn, mx, with);
    for (int k = 0; k < 3; ++k) {
        b.bmn[k] = mn[k];
        b.bsize[k] = mx[k] - mn[k];
        b.c[k] = (mn[k] + mx[k]) * 0.5f;
        b.h[k] = b.bsize[k] * 0.5f;
    }
    b.cascades = opt.n_cascades;
    return b;
}

// Marching box: the outermost cascade (the configured AABB with one cascade).
void Context::fill_aabb(float* mn, float* mx, float* size, const NerfTrainingConfig* with) const {
    base_aabb(mn, mx, with);
    if (opt.n_cascades > 1u) {
        const CascadeBox b = cascade_box(with);
        const float s = std::ldexp(1.0f, static_cast<int>(opt.n_cascades) - 1);
        for (int k = 0; k < 3; ++k) {
            const float hs = b.h[k] * s;
            mn[k] = b.c[k] - hs;
            mx[k] = b.c[k] + hs;
        }
    }
    for (int k = 0; k < 3; ++k) size[k] = mx[k] - mn[k];
}

NerfStatus Context::init(const NerfCreateDesc& d, const NerfB200Options& o) {
    opt = o;
    if (opt.n_levels != 16u) return NERF_STATUS_INVALID_USAGE;  // the fused field takes 16 levels x 2 features
    if (opt.n_cascades == 0u || opt.n_cascades > 8u) return NERF_STATUS_INVALID_USAGE;
    if (grid_layout(opt.n_levels, opt.log2_hashmap_size, opt.base_resolution, opt.max_resolution, &grid) != 0)
        return NERF_STATUS_INVALID_USAGE;
    lt = make_level_table(grid);
    n_grid = 2ull * grid.offset[grid.n_levels];
    n_params = n_grid + kMlpParams;
    n_images = d.image_count;
    width = d.image_width;
    height = d.image_height;
    fx = d.fx;
    fy = d.fy;
    cx = d.cx;
    cy = d.cy;
    grid_res = d.occupancy_grid_res;
    cell_count = grid_res * grid_res * grid_res * opt.n_cascades;  // cascade after cascade
    words = (cell_count + 31u) / 32u;
    max_sample_steps = d.max_sample_steps;
    max_batch_rays = d.max_batch_rays;
    alignment = d.arena_alignment_bytes ? d.arena_alignment_bytes : 256u;
    if (cudaGetDevice(&device) != cudaSuccess) return NERF_STATUS_CUDA_ERROR;
    cudaDeviceProp prop{};
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return NERF_STATUS_CUDA_ERROR;
    if (prop.major < 10) return NERF_STATUS_FAILURE;  // built for sm_100a only
    if (ensure_attributes() != cudaSuccess) return NERF_STATUS_FAILURE;
    if (cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking) != cudaSuccess) return NERF_STATUS_CUDA_ERROR;
    if (cudaHostAlloc(reinterpret_cast<void**>(&stats_host), sizeof(StatsBlock), cudaHostAllocMapped) != cudaSuccess ||
        cudaHostGetDevicePointer(reinterpret_cast<void**>(&stats_host_dev), stats_host, 0) != cudaSuccess)
        return NERF_STATUS_FAILURE;
    *stats_host = StatsBlock{};
    if (cudaEventCreate(&ev0) != cudaSuccess || cudaEventCreate(&ev1) != cudaSuccess) return NERF_STATUS_CUDA_ERROR;

    // model arena
    model.align = std::max<uint64_t>(alignment, 256u);
    const uint64_t o_master = model.add(n_params * 4), o_m = model.add(n_params * 4), o_v = model.add(n_params * 4);
    const uint64_t o_p16 = model.add(n_params * 2), o_gg = model.add(n_grid * 2);
    const uint64_t o_mg = model.add(kMlpGradSlots * 4), o_st = model.add(sizeof(DeviceState));
    const uint64_t o_sync = model.add(sizeof(DpSync)), o_msum = model.add(kMlpGradSlots * 4);
    if (model.alloc() != cudaSuccess) return NERF_STATUS_FAILURE;
    master = model.at<float>(o_master);
    m = model.at<float>(o_m);
    v = model.at<float>(o_v);
    p16 = model.at<__half>(o_p16);
    grid_grad = model.at<__half>(o_gg);
    mlp_grad = model.at<float>(o_mg);
    state = model.at<DeviceState>(o_st);
    dp_sync = model.at<DpSync>(o_sync);
    mlp_sum = model.at<float>(o_msum);
    NB_TRY(cudaMemsetAsync(dp_sync, 0, sizeof(DpSync), stream));

    // occupancy arena
    occ.align = model.align;
    const uint64_t o_den = occ.add(static_cast<uint64_t>(words) * 32u * 4u), o_bits = occ.add(words * 4ull);
    const uint64_t o_full = occ.add(words * 4ull);
    if (occ.alloc() != cudaSuccess) return NERF_STATUS_FAILURE;
    density = occ.at<float>(o_den);
    bitfield = occ.at<uint32_t>(o_bits);
    full_bitfield = occ.at<uint32_t>(o_full);

    // scene arena (reference backend-cuda.cu:1928-1990)
    scene.align = model.align;
    const uint64_t img_bytes = static_cast<uint64_t>(n_images) * width * height * 4u;
    const uint64_t o_img = scene.add(img_bytes), o_cam = scene.add(n_images * 64ull);
    const uint64_t o_inf = scene.add(static_cast<uint64_t>(width) * height * 4u);
    if (scene.alloc() != cudaSuccess) return NERF_STATUS_CUDA_ERROR;
    images = scene.at<uint8_t>(o_img);
    cams = scene.at<float>(o_cam);
    inference_rgba = scene.at<uint32_t>(o_inf);
    if (img_bytes) NB_TRY(cudaMemcpyAsync(images, d.images_rgba8, img_bytes, cudaMemcpyHostToDevice, stream));
    NB_TRY(cudaMemcpyAsync(cams, d.cameras_4x4_packed, n_images * 64ull, cudaMemcpyHostToDevice, stream));
    NB_TRY(cudaMemsetAsync(inference_rgba, 0, static_cast<uint64_t>(width) * height * 4u, stream));

    // parameters: hash table U(-s, s) (its splitmix stream drawn on the device,
    // one thread per value), MLPs with the reference's Xavier draw
    std::vector<float> host(kMlpParams);
    NB_TRY(launch_splitmix_fill(master, n_grid, SplitMix(0x2468ull, 0x1357ull).state, opt.hash_init_scale, stream));
    float* mlp = host.data();
    SplitMix dens(0x1234ull, 0x5678ull);
    xavier(dens, 32, 64, mlp + kMlpD0);
    xavier(dens, 64, 16, mlp + kMlpD1);
    SplitMix col(0x9abcull, 0xdef0ull);
    xavier(col, 32, 64, mlp + kMlpC0);
    xavier(col, 64, 64, mlp + kMlpC1);
    xavier(col, 64, 16, mlp + kMlpC2);
    NB_TRY(cudaMemcpyAsync(master + n_grid, host.data(), kMlpParams * 4, cudaMemcpyHostToDevice, stream));
    NB_TRY(launch_f32_to_f16(master, p16, n_params, stream));
    NB_TRY(cudaMemsetAsync(m, 0, n_params * 4, stream));
    NB_TRY(cudaMemsetAsync(v, 0, n_params * 4, stream));
    NB_TRY(cudaMemsetAsync(grid_grad, 0, n_grid * 2, stream));
    NB_TRY(cudaMemsetAsync(mlp_grad, 0, kMlpGradSlots * 4, stream));
    NB_TRY(cudaMemsetAsync(state, 0, sizeof(DeviceState), stream));
    NB_TRY(cudaMemsetAsync(density, 0, static_cast<uint64_t>(words) * 32u * 4u, stream));
    NB_TRY(cudaMemsetAsync(bitfield, 0, words * 4ull, stream));
    NB_TRY(cudaMemsetAsync(full_bitfield, 0xFF, words * 4ull, stream));
    NB_TRY(cudaStreamSynchronize(stream));
    return NERF_STATUS_OK;
}

NerfStatus Context::configure(const NerfTrainingConfig& c) {
    // Validation of the reference (backend-cuda.cu:2137-2140); the per-ray step
    // limit is 4096 here instead of 256.  With a per-step sample target or cap
    // the stream is capacity-bounded instead of rays x steps.
    const uint64_t total = static_cast<uint64_t>(c.rays_per_batch) * c.max_sample_steps_per_ray;
    if (c.rays_per_batch == 0u || c.max_sample_steps_per_ray == 0u || c.max_sample_steps_per_ray > kMaxStepsPerRay)
        return NERF_STATUS_INVALID_USAGE;
    if (c.occupancy_params.update_interval == 0u || n_images == 0u) return NERF_STATUS_INVALID_USAGE;
    if (c.rays_per_batch > max_batch_rays) return NERF_STATUS_INVALID_USAGE;
    if (!(c.aabb_max_x > c.aabb_min_x && c.aabb_max_y > c.aabb_min_y && c.aabb_max_z > c.aabb_min_z))
        return NERF_STATUS_INVALID_USAGE;
    if (!(c.hyper_params.loss_scale > 0.0f)) return NERF_STATUS_INVALID_USAGE;
    const bool bounded = opt.target_samples_per_step != 0u || opt.max_samples_per_step != 0u;
    uint64_t cap;
    if (bounded) {
        // The documented rule (NerfB200Options::max_samples_per_step): an
        // explicit cap, else rays x steps, within the sample buffers.
        cap = opt.max_samples_per_step ? opt.max_samples_per_step : total;
        cap = std::min<uint64_t>(cap, max_sample_steps);
    } else {
        if (total > max_sample_steps || total > 0xFFFFFFFFull) return NERF_STATUS_INVALID_USAGE;
        cap = total;
    }
    if (cudaStreamSynchronize(stream) != cudaSuccess) return NERF_STATUS_CUDA_ERROR;
    release_graph();
    configured = false;
    cfg = c;

    TrainConsts& t = tc;
    t = TrainConsts{};
    t.n_images = n_images;
    t.width = width;
    t.height = height;
    t.fx = fx;
    t.fy = fy;
    t.cx = cx;
    t.cy = cy;
    fill_aabb(t.aabb_min, t.aabb_max, t.aabb_size, &c);  // the new configuration's box (outermost cascade)
    t.casc = cascade_box(&c);
    const float ifx = fx > 0.0f ? 1.0f / fx : 0.0f, ify = fy > 0.0f ? 1.0f / fy : 0.0f;
    t.cone = 0.5f * (ifx + ify);
    t.max_rays = max_batch_rays;
    t.max_steps = c.max_sample_steps_per_ray;
    t.mask_words = (c.max_sample_steps_per_ray + 31u) / 32u;
    t.sample_cap = static_cast<uint32_t>(cap);
    t.rays_per_batch = c.rays_per_batch;
    t.dp_rank = dp_rank;
    t.dp_world = dp_world;
    t.background = opt.background;
    t.target_samples = opt.target_samples_per_step;
    t.grid_res = grid_res;
    t.cell_count = cell_count;
    t.update_count = std::min(c.occupancy_params.cells_per_update, cell_count);
    t.warmup_steps = c.occupancy_params.warmup_steps;
    t.update_interval = c.occupancy_params.update_interval;
    t.occ_decay = c.occupancy_params.decay;
    t.occ_threshold = c.occupancy_params.threshold;
    t.loss_scale = c.hyper_params.loss_scale;
    t.stop_transmittance = opt.stop_transmittance;
    t.lr = c.hyper_params.learning_rate;
    t.beta1 = c.hyper_params.adam_beta1;
    t.beta2 = c.hyper_params.adam_beta2;
    t.eps = c.hyper_params.adam_eps;
    t.clip = c.hyper_params.grad_clip_norm;
    t.guard = c.hyper_params.update_guard_grad_norm;
    t.lr_decay_ksteps = c.hyper_params.lr_decay_ksteps;

    // batch arena
    mlp_tc = env_u32("NERF_B200_MLP_TC", 0u) != 0u && mlp_backward_tc_blocks() != 0u;
    n_partials = mlp_tc ? mlp_backward_tc_blocks() : field_backward_blocks();
    fwd_blocks = field_forward_blocks();
    batch.align = model.align;
    batch.size = 0;
    const uint64_t o_rc = batch.add(2ull * t.max_rays * 4ull), o_kept = batch.add(static_cast<uint64_t>(t.max_steps) * t.max_rays * 4u);
    const uint64_t o_st = batch.add(static_cast<uint64_t>(t.mask_words) * t.max_rays * 4u);
    const uint64_t o_geom = batch.add(t.max_rays * sizeof(RayGeom));
    const uint64_t o_bs = batch.add(t.max_rays * 4ull), o_ba = batch.add(t.max_rays * 4ull);
    const uint64_t o_rays = batch.add(t.max_rays * sizeof(RayRecord)), o_ri = batch.add(t.max_rays * 4ull);
    const uint64_t o_pos = batch.add(cap * 16u), o_sr = batch.add(cap * 4u), o_feat = batch.add(cap * 112u);
    const uint64_t o_raw = batch.add(cap * 16u), o_dout = batch.add(cap * 16u), o_dfeat = batch.add(cap * 64u);
    const uint64_t o_part = batch.add(static_cast<uint64_t>(n_partials) * kMlpParams * 4u);
    const uint64_t o_sig = batch.add(std::max<uint32_t>(t.update_count, 1u) * 4ull);
    const uint64_t own_max = dp_peer ? ((n_grid / 8u + dp_world - 1u) / dp_world + 1u) * 8u : 1u;
    const uint64_t o_gsum = batch.add(own_max * 4u);
    if (batch.alloc() != cudaSuccess) return NERF_STATUS_FAILURE;
    ray_counts = batch.at<uint32_t>(o_rc);
    kept_t = batch.at<float>(o_kept);
    chunk_t = batch.at<float>(o_st);
    geom = batch.at<RayGeom>(o_geom);
    ray_offset = batch.at<uint32_t>(o_bs);
    ray_slot = batch.at<uint32_t>(o_ba);
    rays = batch.at<RayRecord>(o_rays);
    ray_index = batch.at<uint32_t>(o_ri);
    pos_dt = batch.at<float4>(o_pos);
    sample_ray = batch.at<uint32_t>(o_sr);
    feat = batch.at<void>(o_feat);
    raw = batch.at<float4>(o_raw);
    dout = batch.at<float4>(o_dout);
    dfeat = batch.at<void>(o_dfeat);
    partials = batch.at<float>(o_part);
    occ_sigma = batch.at<float>(o_sig);
    dp_gsum = batch.at<float>(o_gsum);
    NB_TRY(cudaMemsetAsync(batch.base, 0, batch.size, stream));

    // Fresh optimiser / occupancy / step state (reference backend-cuda.cu:2205-2215).
    DeviceState st{};
    st.n_rays = c.rays_per_batch;
    NB_TRY(cudaMemcpyAsync(state, &st, sizeof(st), cudaMemcpyHostToDevice, stream));
    stats_host_current = false;
    NB_TRY(cudaMemsetAsync(density, 0, static_cast<uint64_t>(words) * 32u * 4u, stream));
    NB_TRY(cudaMemsetAsync(bitfield, 0, words * 4ull, stream));
    NB_TRY(cudaMemsetAsync(m, 0, n_params * 4, stream));
    NB_TRY(cudaMemsetAsync(v, 0, n_params * 4, stream));
    NB_TRY(cudaMemsetAsync(grid_grad, 0, n_grid * 2, stream));
    NB_TRY(cudaMemsetAsync(mlp_grad, 0, kMlpGradSlots * 4, stream));
    NB_TRY(launch_march(sampler_args(), stream));  // the first step's march; later ones run inside the steps
    configured = true;
    occupancy_valid = false;
    host_generation = 0;
    const NerfStatus s = capture_graph();
    if (s != NERF_STATUS_OK) {
        configured = false;
        return s;
    }
    if (cudaStreamSynchronize(stream) != cudaSuccess) return NERF_STATUS_CUDA_ERROR;
    return NERF_STATUS_OK;
}

SamplerArgs Context::sampler_args() const {
    SamplerArgs sa{};
    sa.tc = tc;
    sa.state = state;
    sa.cams = cams;
    sa.images = images;
    sa.bitfield = bitfield;
    sa.ray_counts = ray_counts;
    sa.kept_t = kept_t;
    sa.chunk_t = chunk_t;
    sa.geom = geom;
    sa.ray_offset = ray_offset;
    sa.ray_slot = ray_slot;
    sa.rays = rays;
    sa.pos_dt = pos_dt;
    sa.sample_ray = sample_ray;
    sa.ray_index = ray_index;
    return sa;
}

// The kernels of one training step, in order.  The captured graph and the
// profiled (eager, event-timed) step both come from here, so they cannot
// diverge.  ev: optional events recorded before the first and after every
// kernel (kStepKernels + 1 of them).
cudaError_t Context::enqueue_step(cudaStream_t s, cudaEvent_t* ev) {
    FieldArgs occq = field_args();
    occq.grid_res = grid_res;
    occq.cell_count = cell_count;
    occq.update_count = tc.update_count;
    occq.warmup_steps = tc.warmup_steps;
    occq.update_interval = tc.update_interval;
    occq.occ_sigma = occ_sigma;

    OccupancyArgs oa{};
    oa.state = state;
    oa.density = density;
    oa.bitfield = bitfield;
    oa.occ_sigma = occ_sigma;
    oa.cell_count = cell_count;
    oa.update_count = tc.update_count;
    oa.warmup_steps = tc.warmup_steps;
    oa.update_interval = tc.update_interval;
    oa.decay = tc.occ_decay;
    oa.threshold = tc.occ_threshold;

    const SamplerArgs sa = sampler_args();

    FieldArgs fa = field_args();
    fa.pos_dt = pos_dt;
    fa.sample_ray = sample_ray;
    fa.rays = rays;
    fa.feat = feat;
    fa.raw = raw;
    fa.dout = dout;
    fa.grid_grad = grid_grad;
    fa.partials = partials;
    fa.dfeat = dfeat;

    CompositeArgs ca{};
    ca.rays = rays;
    ca.raw = raw;
    ca.pos_dt = pos_dt;
    ca.dout = dout;
    ca.state = state;
    ca.loss_slot = mlp_grad + kMlpGradLoss;
    ca.max_rays = tc.max_rays;
    ca.dp_world = dp_world;
    ca.loss_scale = tc.loss_scale;
    ca.stop_transmittance = tc.stop_transmittance;

    OptimArgs op{};
    op.tc = tc;
    op.state = state;
    op.master = master;
    op.params16 = p16;
    op.grid_grad = grid_grad;
    op.mlp_grad = mlp_grad;
    op.m = m;
    op.v = v;
    op.partials = partials;
    op.n_partials = n_partials;
    op.n_grid = n_grid;
    op.n_params = n_params;
    op.stats_blocks = grad_stats_blocks(n_params, !dp_active());
    op.mlp_in = mlp_grad;
    op.world = dp_world;
    if (dp_peer) {
        op.dp_peer = 1u;
        op.dp = dp_peers();
        op.mlp_in = mlp_sum;
    }

    cudaError_t e;
    int k = 0;
    auto mark = [&]() -> cudaError_t { return ev ? cudaEventRecord(ev[k++], s) : cudaSuccess; };
    if ((e = mark()) != cudaSuccess) return e;
    if ((e = launch_field_forward(occq, kFieldOccupancy, fwd_blocks, s)) != cudaSuccess || (e = mark()) != cudaSuccess) return e;
    if ((e = launch_occupancy_update(oa, s)) != cudaSuccess || (e = mark()) != cudaSuccess) return e;
    if ((e = launch_sample_bits(sa, s)) != cudaSuccess || (e = mark()) != cudaSuccess) return e;
    if ((e = launch_sample_scan(sa, s)) != cudaSuccess || (e = mark()) != cudaSuccess) return e;
    if ((e = launch_sample_write(sa, s)) != cudaSuccess || (e = mark()) != cudaSuccess) return e;
    if (mlp_tc) {  // encode + SH into the training rows, then the MLPs on tcgen05
        if ((e = launch_field_encode(fa, s)) != cudaSuccess ||
            (e = launch_mlp_forward_tc_train(p16 + n_grid, feat, &state->n_samples, reinterpret_cast<float*>(raw), &state->mlp_error,
                                             s)) != cudaSuccess)
            return e;
    } else if ((e = launch_field_forward(fa, kFieldTrain, fwd_blocks, s)) != cudaSuccess) {
        return e;
    }
    if ((e = mark()) != cudaSuccess) return e;
    if ((e = launch_composite(ca, s)) != cudaSuccess || (e = mark()) != cudaSuccess) return e;
    // MLP backward (writes the feature gradients), then the hash-table scatter.
    if (mlp_tc) {  // on tcgen05
        if ((e = launch_mlp_backward_tc(p16 + n_grid, feat, 1, nullptr, reinterpret_cast<const float*>(dout), &state->n_samples, 0u,
                                        dfeat, partials, n_partials, &state->mlp_error, s)) != cudaSuccess)
            return e;
    } else if ((e = launch_field_backward(fa, kFieldTrain, n_partials, s)) != cudaSuccess) {
        return e;
    }
    if ((e = mark()) != cudaSuccess) return e;
    if ((e = launch_grid_scatter(fa, s)) != cudaSuccess || (e = mark()) != cudaSuccess) return e;
    // One GPU: the statistics kernel also reduces the weight-gradient partials.
    op.fuse_wgrad = dp_active() ? 0u : 1u;
    op.stats_host = stats_host_dev;
    if (!op.fuse_wgrad && (e = launch_wgrad_reduce(op, s)) != cudaSuccess) return e;
    if ((e = mark()) != cudaSuccess) return e;
    if (dp_peer) {
        // Peer mode, no collective library in the step: after a barrier (every
        // rank's gradients are complete) each rank sums its owned range of all
        // ranks' hash gradients and all ranks' MLP gradients over NVLink and
        // publishes its owned range's sum of squares; after a second barrier
        // (every rank has read this rank's gradients) they are cleared.
        if ((e = launch_dp_barrier(op.dp, s)) != cudaSuccess || (e = launch_dp_reduce_grads(op, s)) != cudaSuccess ||
            (e = launch_dp_barrier(op.dp, s)) != cudaSuccess ||
            (e = cudaMemsetAsync(grid_grad, 0, n_grid * 2u, s)) != cudaSuccess)
            return e;
    } else if (comm) {
        if (g_nccl.all_reduce(grid_grad, grid_grad, n_grid, ncclFloat16, ncclSum, comm, s) != ncclSuccess ||
            g_nccl.all_reduce(mlp_grad, mlp_grad, kMlpGradSlots, ncclFloat32, ncclSum, comm, s) != ncclSuccess)
            return cudaErrorUnknown;
    }
    if ((e = mark()) != cudaSuccess) return e;
    if ((e = launch_grad_stats(op, s)) != cudaSuccess || (e = mark()) != cudaSuccess) return e;
    // The statistics kernel advanced the frame and set the next ray count:
    // the next step's march.  (Run beside Adam on a second stream it gained
    // nothing: with HBM saturated by Adam the march's stores stall, and the
    // pair took longer than the two in order.)
    if ((e = launch_march(sa, s)) != cudaSuccess || (e = mark()) != cudaSuccess || (e = launch_adam(op, s)) != cudaSuccess)
        return e;
    // Peer mode: every rank wrote its owned fp16 parameters into every rank's
    // mirror; no rank reads them before all writes are done.
    if (dp_peer && (e = launch_dp_barrier(op.dp, s)) != cudaSuccess) return e;
    if ((e = mark()) != cudaSuccess) return e;
    return cudaSuccess;
}

// Maps every rank's model arena into this process (CUDA IPC; handles
// exchanged with an NCCL all-gather).  All ranks agree on the result through a
// min all-reduce, so either all use peer mode or all keep the all-reduce path.
NerfStatus Context::open_peers() {
    const char* env = std::getenv("NERF_B200_DP_PEER");
    bool want = dp_world <= kMaxDpWorld && !(env && env[0] == '0');
    const size_t hb = sizeof(cudaIpcMemHandle_t);
    cudaIpcMemHandle_t mine{};
    if (want && cudaIpcGetMemHandle(&mine, model.base) != cudaSuccess) {
        cudaGetLastError();
        want = false;
    }
    unsigned char* dbuf = nullptr;
    if (cudaMalloc(&dbuf, hb * (dp_world + 1u) + 16u) != cudaSuccess) return NERF_STATUS_FAILURE;
    std::vector<unsigned char> all(hb * dp_world);
    float* flag = reinterpret_cast<float*>(dbuf + hb * (dp_world + 1u));
    bool ok = cudaMemcpy(dbuf + hb * dp_world, &mine, hb, cudaMemcpyHostToDevice) == cudaSuccess &&
              g_nccl.all_gather(dbuf + hb * dp_world, dbuf, hb, ncclUint8, comm, stream) == ncclSuccess &&
              cudaStreamSynchronize(stream) == cudaSuccess &&
              cudaMemcpy(all.data(), dbuf, hb * dp_world, cudaMemcpyDeviceToHost) == cudaSuccess;
    bool opened = ok && want;
    if (opened) {
        std::vector<unsigned char> full(kDpHandleBytes * dp_world, 0);
        for (uint32_t r = 0; r < dp_world; ++r) std::memcpy(full.data() + kDpHandleBytes * r, all.data() + hb * r, hb);
        opened = map_peers(full.data());
    }
    const float f = opened ? 1.0f : 0.0f;
    float agreed = 0.0f;
    ok = ok && cudaMemcpy(flag, &f, 4, cudaMemcpyHostToDevice) == cudaSuccess &&
         g_nccl.all_reduce(flag, flag, 1, ncclFloat32, ncclMin, comm, stream) == ncclSuccess &&
         cudaStreamSynchronize(stream) == cudaSuccess && cudaMemcpy(&agreed, flag, 4, cudaMemcpyDeviceToHost) == cudaSuccess;
    cudaFree(dbuf);
    dp_peer = ok && agreed > 0.5f;
    if (!dp_peer) {
        for (uint32_t r = 0; r < kMaxDpWorld; ++r)
            if (peer_model[r] && r != dp_rank) cudaIpcCloseMemHandle(peer_model[r]);
        for (auto& p : peer_model) p = nullptr;
    }
    return ok ? NERF_STATUS_OK : NERF_STATUS_FAILURE;
}

bool Context::map_peers(const unsigned char* handles) {
    bool opened = true;
    for (uint32_t r = 0; r < dp_world && opened; ++r) {
        if (r == dp_rank) {
            peer_model[r] = model.base;
            continue;
        }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, handles + kDpHandleBytes * r, sizeof(h));
        void* p = nullptr;
        if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            opened = false;
            break;
        }
        peer_model[r] = static_cast<unsigned char*>(p);
    }
    if (!opened) {
        for (uint32_t r = 0; r < kMaxDpWorld; ++r)
            if (peer_model[r] && r != dp_rank) cudaIpcCloseMemHandle(peer_model[r]);
        for (auto& p : peer_model) p = nullptr;
    }
    return opened;
}

DpPeers Context::dp_peers() const {
    DpPeers d{};
    d.world = dp_world;
    d.rank = dp_rank;
    d.lo = dp_lo(dp_rank);
    d.hi = dp_lo(dp_rank + 1u);
    for (uint32_t r = 0; r < dp_world; ++r) {
        d.grad[r] = peer(r, grid_grad);
        d.mlp[r] = peer(r, mlp_grad);
        d.p16[r] = peer(r, p16);
        d.sync[r] = peer(r, dp_sync);
    }
    d.gsum = dp_gsum;
    d.mlp_sum = mlp_sum;
    d.timeout_ns = dp_timeout_ns;
    return d;
}

cudaError_t Context::read_sharded(void* host, const float* local, uint64_t n) const {
    if (!dp_peer) return cudaMemcpy(host, local, n * 4u, cudaMemcpyDeviceToHost);
    float* h = static_cast<float*>(host);
    for (uint32_t r = 0; r < dp_world; ++r) {
        const uint64_t lo = dp_lo(r), hi = dp_lo(r + 1u);
        const cudaError_t e = cudaMemcpy(h + lo, peer(r, local) + lo, (hi - lo) * 4u, cudaMemcpyDefault);
        if (e != cudaSuccess) return e;
    }
    return n > n_grid ? cudaMemcpy(h + n_grid, local + n_grid, (n - n_grid) * 4u, cudaMemcpyDeviceToHost) : cudaSuccess;
}

NerfStatus Context::capture_graph() {
    if (cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) return NERF_STATUS_CUDA_ERROR;
    const cudaError_t e = enqueue_step(stream, nullptr);
    cudaGraph_t g = nullptr;
    const cudaError_t ee = cudaStreamEndCapture(stream, &g);
    if (e != cudaSuccess || ee != cudaSuccess || !g) {
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        return NERF_STATUS_CUDA_ERROR;
    }
    graph = g;
    if (cudaGraphInstantiate(&exec, graph, nullptr, nullptr, 0) != cudaSuccess) return NERF_STATUS_CUDA_ERROR;
    if (cudaGraphUpload(exec, stream) != cudaSuccess) return NERF_STATUS_CUDA_ERROR;
    return NERF_STATUS_OK;
}

NerfStatus Context::ensure_render_buffers(uint32_t w, uint32_t h) {
    if (render.base && render_w == w && render_h == h) return NERF_STATUS_OK;
    render.release();
    render.size = 0;
    render.align = model.align;
    const uint64_t o_rgba = render.add(static_cast<uint64_t>(w) * h * 4u), o_cnt = render.add(16), o_tot = render.add(16);
    if (render.alloc() != cudaSuccess) return NERF_STATUS_FAILURE;
    render_rgba = render.at<uint32_t>(o_rgba);
    render_counter = render.at<uint32_t>(o_cnt);
    render_samples = render.at<unsigned long long>(o_tot);
    render_w = w;
    render_h = h;
    return NERF_STATUS_OK;
}

NerfStatus Context::render_view(const float* c2w, uint32_t w, uint32_t h, float fx_, float fy_, float cx_, float cy_,
                                uint32_t max_steps, float stop, uint32_t tile, uint32_t rank, uint32_t world,
                                NerfB200RenderInfo* info) {
    if (w == 0u || h == 0u || max_steps == 0u) return NERF_STATUS_INVALID_USAGE;
    if (tile != 0u && (world == 0u || rank >= world)) return NERF_STATUS_INVALID_USAGE;
    const NerfStatus s = ensure_render_buffers(w, h);
    if (s != NERF_STATUS_OK) return s;
    RenderArgs ra{};
    ra.lt = lt;
    ra.params16 = p16;
    ra.mlp_offset = static_cast<uint32_t>(n_grid);
    ra.bitfield = occupancy_valid ? bitfield : full_bitfield;
    ra.grid_res = grid_res;
    fill_aabb(ra.aabb_min, ra.aabb_max, ra.aabb_size);
    ra.casc = cascade_box();
    std::memcpy(ra.c2w, c2w, 12 * sizeof(float));
    ra.width = w;
    ra.height = h;
    ra.fx = fx_;
    ra.fy = fy_;
    ra.cx = cx_;
    ra.cy = cy_;
    ra.max_steps = max_steps;
    ra.stop_transmittance = stop;
    ra.tile = tile;
    ra.tile_rank = rank;
    ra.tile_world = world ? world : 1u;
    ra.rgba = render_rgba;
    ra.work_counter = render_counter;
    ra.total_samples = render_samples;
    NB_TRY(cudaMemsetAsync(render_counter, 0, 16, stream));
    NB_TRY(cudaMemsetAsync(render_samples, 0, 16, stream));
    NB_TRY(cudaEventRecord(ev0, stream));
    NB_TRY(launch_render(ra, stream));
    NB_TRY(cudaEventRecord(ev1, stream));
    if (info) {
        unsigned long long samples = 0;
        NB_TRY(cudaMemcpyAsync(&samples, render_samples, 8, cudaMemcpyDeviceToHost, stream));
        NB_TRY(cudaStreamSynchronize(stream));
        float ms = 0.0f;
        NB_TRY(cudaEventElapsedTime(&ms, ev0, ev1));
        uint64_t rays_n = static_cast<uint64_t>(w) * h;
        if (tile != 0u) {
            const uint32_t tx = (w + tile - 1u) / tile, ty = (h + tile - 1u) / tile;
            rays_n = 0;
            for (uint32_t t = rank; t < tx * ty; t += world) {
                const uint32_t x0 = (t % tx) * tile, y0 = (t / tx) * tile;
                rays_n += static_cast<uint64_t>(std::min(tile, w - x0)) * std::min(tile, h - y0);
            }
        }
        info->rays = rays_n;
        info->samples = samples;
        info->milliseconds = ms;
    }
    return NERF_STATUS_OK;
}

// ------------------------------------------------------- checkpoint format
// u64 little-endian header length, JSON header, fp32 tensors back to back
// (the container of reference backend-cuda.cu:2466-2525).  Tensors: the MLP
// matrices under the reference's naming scheme and the hash table as
// "encoding.hash_grid" [entries, 2].
namespace ckpt {
struct Tensor {
    std::string name;
    uint32_t rows, cols;
    uint64_t offset;  // into the flat parameter vector
};
std::vector<Tensor> layout(uint64_t n_grid) {
    std::vector<Tensor> t;
    t.push_back({"encoding.hash_grid", static_cast<uint32_t>(n_grid / 2u), 2u, 0u});
    t.push_back({"density.input.weight", 64u, 32u, n_grid + kMlpD0});
    t.push_back({"density.output.weight", 16u, 64u, n_grid + kMlpD1});
    t.push_back({"color.input.weight", 64u, 32u, n_grid + kMlpC0});
    t.push_back({"color.hidden.0.weight", 64u, 64u, n_grid + kMlpC1});
    t.push_back({"color.output.weight", 16u, 64u, n_grid + kMlpC2});
    return t;
}

// Minimal reader for the header this writer produces: an object of objects
// whose "data_offsets" / "shape" are integer arrays.
struct Json {
    const std::string& s;
    size_t i = 0;
    explicit Json(const std::string& str) : s(str) {}
    void ws() {
        while (i < s.size() && (s[i] == ' ' || s[i] == '\n' || s[i] == '\t' || s[i] == '\r')) ++i;
    }
    bool expect(char c) {
        ws();
        if (i < s.size() && s[i] == c) {
            ++i;
            return true;
        }
        return false;
    }
    bool string(std::string& out) {
        ws();
        if (i >= s.size() || s[i] != '"') return false;
        ++i;
        out.clear();
        while (i < s.size() && s[i] != '"') {
            if (s[i] == '\\' && i + 1 < s.size()) ++i;
            out.push_back(s[i++]);
        }
        if (i >= s.size()) return false;
        ++i;
        return true;
    }
    bool skip_value() {
        ws();
        if (i >= s.size()) return false;
        const char c = s[i];
        if (c == '"') {
            std::string tmp;
            return string(tmp);
        }
        if (c == '{' || c == '[') {
            const char close = c == '{' ? '}' : ']';
            ++i;
            ws();
            if (i < s.size() && s[i] == close) {
                ++i;
                return true;
            }
            for (;;) {
                if (c == '{') {
                    std::string k;
                    if (!string(k) || !expect(':')) return false;
                }
                if (!skip_value()) return false;
                ws();
                if (i < s.size() && s[i] == ',') {
                    ++i;
                    continue;
                }
                return expect(close);
            }
        }
        while (i < s.size() && s[i] != ',' && s[i] != '}' && s[i] != ']') ++i;
        return true;
    }
    bool int_array(std::vector<uint64_t>& out) {
        out.clear();
        if (!expect('[')) return false;
        ws();
        if (i < s.size() && s[i] == ']') {
            ++i;
            return true;
        }
        for (;;) {
            ws();
            size_t j = i;
            while (j < s.size() && s[j] >= '0' && s[j] <= '9') ++j;
            if (j == i) return false;
            out.push_back(std::strtoull(s.substr(i, j - i).c_str(), nullptr, 10));
            i = j;
            ws();
            if (i < s.size() && s[i] == ',') {
                ++i;
                continue;
            }
            return expect(']');
        }
    }
};
struct Entry {
    std::vector<uint64_t> shape, offsets;
};
bool parse(const std::string& header, std::map<std::string, Entry>& out) {
    Json j(header);
    if (!j.expect('{')) return false;
    j.ws();
    if (j.i < header.size() && header[j.i] == '}') return true;
    for (;;) {
        std::string key;
        if (!j.string(key) || !j.expect(':')) return false;
        if (key == "__metadata__") {
            if (!j.skip_value()) return false;
        } else {
            if (!j.expect('{')) return false;
            Entry e;
            for (;;) {
                std::string f;
                if (!j.string(f) || !j.expect(':')) return false;
                if (f == "shape") {
                    if (!j.int_array(e.shape)) return false;
                } else if (f == "data_offsets") {
                    if (!j.int_array(e.offsets)) return false;
                } else if (!j.skip_value()) {
                    return false;
                }
                if (j.expect(',')) continue;
                if (!j.expect('}')) return false;
                break;
            }
            out[key] = e;
        }
        if (j.expect(',')) continue;
        return j.expect('}');
    }
}
}  // namespace ckpt

Context* as_ctx(void* p) { return static_cast<Context*>(p); }

}  // namespace nb

using nb::Context;
using nb::as_ctx;

// =================================================================== nerf.h
extern "C" {

NERF_API void nerf_b200_default_options(NerfB200Options* o) {
    if (!o) return;
    o->n_levels = 16;
    o->log2_hashmap_size = nb::env_u32("NERF_B200_LOG2_HASHMAP_SIZE", 19u);
    o->base_resolution = nb::env_u32("NERF_B200_BASE_RESOLUTION", 16u);
    o->max_resolution = nb::env_u32("NERF_B200_MAX_RESOLUTION", 2048u);
    o->hash_init_scale = 1e-4f;
    o->background = nb::env_u32("NERF_B200_BACKGROUND", 0u);
    o->stop_transmittance = nb::env_float("NERF_B200_STOP_T", 1e-4f);
    o->render_stop_transmittance = nb::env_float("NERF_B200_RENDER_STOP_T", 1e-4f);
    o->target_samples_per_step = nb::env_u32("NERF_B200_TARGET_SAMPLES", 0u);
    o->max_samples_per_step = nb::env_u32("NERF_B200_MAX_SAMPLES", 0u);
    o->n_cascades = nb::env_u32("NERF_B200_CASCADES", 1u);
}

NERF_API NerfStatus nerf_b200_create_context(const NerfCreateDesc* desc, const NerfB200Options* options, void** out) {
    if (!desc || !out || !options) return NERF_STATUS_INVALID_USAGE;
    *out = nullptr;
    const NerfCreateDesc d = *desc;
    if (d.arena_alignment_bytes != 0u && (d.arena_alignment_bytes & (d.arena_alignment_bytes - 1u)) != 0u)
        return NERF_STATUS_INVALID_USAGE;
    if (d.occupancy_grid_res == 0u || d.occupancy_grid_res > 1024u || d.max_batch_rays == 0u) return NERF_STATUS_INVALID_USAGE;
    if (d.image_count != 0u && (!d.images_rgba8 || !d.cameras_4x4_packed)) return NERF_STATUS_INVALID_USAGE;
    const uint64_t need_img = static_cast<uint64_t>(d.image_count) * d.image_width * d.image_height * 4u;
    if (d.images_bytes < need_img || d.cameras_bytes < d.image_count * 64ull) return NERF_STATUS_INVALID_USAGE;
    std::unique_ptr<Context> c(new (std::nothrow) Context());
    if (!c) return NERF_STATUS_FAILURE;
    try {
        const NerfStatus s = c->init(d, *options);
        if (s != NERF_STATUS_OK) return s;
    } catch (...) {
        return NERF_STATUS_FAILURE;
    }
    *out = c.release();
    return NERF_STATUS_OK;
}

NERF_API NerfStatus nerf_create_context(const NerfCreateDesc* desc, void** out_context) {
    NerfB200Options o;
    nerf_b200_default_options(&o);
    return nerf_b200_create_context(desc, &o, out_context);
}

NERF_API NerfStatus nerf_destroy_context(void* context) {
    if (!context) return NERF_STATUS_OK;
    Context* c = as_ctx(context);
    {
        std::lock_guard<std::mutex> lk(c->mu);
        c->release_all();
    }
    delete c;
    return NERF_STATUS_OK;
}

NERF_API NerfStatus nerf_configure_training(void* context, const NerfTrainingConfig* config) {
    if (!context || !config) return NERF_STATUS_INVALID_USAGE;
    Context* c = as_ctx(context);
    std::lock_guard<std::mutex> lk(c->mu);
    try {
        return c->configure(*config);
    } catch (...) {
        return NERF_STATUS_FAILURE;
    }
}

NERF_API NerfStatus nerf_train_step(void* context) {
    if (!context) return NERF_STATUS_INVALID_USAGE;
    Context* c = as_ctx(context);
    std::lock_guard<std::mutex> lk(c->mu);
    if (!c->configured || !c->exec) return NERF_STATUS_STATE_ERROR;
    if (cudaGraphLaunch(c->exec, c->stream) != cudaSuccess) return NERF_STATUS_CUDA_ERROR;
    ++c->host_generation;
    c->stats_host_current = true;
    c->occupancy_valid = true;
    return NERF_STATUS_OK;
}

NERF_API NerfStatus nerf_read_train_stats(void* context, NerfTrainStats* out) {
    if (!context || !out) return NERF_STATUS_INVALID_USAGE;
    Context* c = as_ctx(context);
    std::lock_guard<std::mutex> lk(c->mu);
    if (!c->configured) return NERF_STATUS_STATE_ERROR;
    const bool mirror = c->stats_host_current;
    if (!mirror) NB_TRY(cudaMemcpyAsync(out, &c->state->stats, sizeof(NerfTrainStats), cudaMemcpyDeviceToHost, c->stream));
    uint32_t dp_error = 0u, mlp_error = 0u;
    if (c->dp_peer || c->dp_watch) NB_TRY(cudaMemcpyAsync(&dp_error, &c->dp_sync->error, 4, cudaMemcpyDeviceToHost, c->stream));
    if (c->mlp_tc) NB_TRY(cudaMemcpyAsync(&mlp_error, &c->state->mlp_error, 4, cudaMemcpyDeviceToHost, c->stream));
    NB_TRY(cudaStreamSynchronize(c->stream));
    if (mirror) {
        const volatile nb::StatsBlock* h = c->stats_host;
        out->loss = h->loss;
        out->grad_norm = h->grad_norm;
        out->has_nonfinite = h->has_nonfinite;
        out->completed_steps = h->completed_steps;
        out->last_train_camera = h->last_train_camera;
    }
    c->host_generation = out->completed_steps;
    // A data-parallel barrier that timed out (a rank stopped stepping): the
    // replicas are no longer in step.  A tensor-core MLP kernel whose MMAs did
    // not complete: the step's gradients are incomplete.
    return (dp_error || mlp_error) ? NERF_STATUS_CUDA_ERROR : NERF_STATUS_OK;
}

NERF_API NerfStatus nerf_inference(void* context, const NerfInferenceRequest* req, NerfInferenceInfo* info) {
    if (!context || !req) return NERF_STATUS_INVALID_USAGE;
    Context* c = as_ctx(context);
    std::lock_guard<std::mutex> lk(c->mu);
    if (req->samples_per_ray == 0u || req->camera_idx >= c->n_images) return NERF_STATUS_INVALID_USAGE;
    const uint64_t bytes = static_cast<uint64_t>(c->width) * c->height * 4u;
    if (req->dst_rgba8 && req->dst_bytes < bytes) return NERF_STATUS_INVALID_USAGE;
    if (req->dst_rgba8 && req->memory_kind != NERF_MEMORY_HOST && req->memory_kind != NERF_MEMORY_CUDA_DEVICE)
        return NERF_STATUS_INVALID_USAGE;
    float cam[16];
    NB_TRY(cudaMemcpyAsync(cam, c->cams + 16ull * req->camera_idx, 64, cudaMemcpyDeviceToHost, c->stream));
    NB_TRY(cudaStreamSynchronize(c->stream));
    const NerfStatus s = c->render_view(cam, c->width, c->height, c->fx, c->fy, c->cx, c->cy, req->samples_per_ray,
                                        c->opt.render_stop_transmittance, 0, 0, 1, nullptr);
    if (s != NERF_STATUS_OK) return s;
    NB_TRY(cudaMemcpyAsync(c->inference_rgba, c->render_rgba, bytes, cudaMemcpyDeviceToDevice, c->stream));
    if (req->dst_rgba8) {
        const cudaMemcpyKind kind = req->memory_kind == NERF_MEMORY_CUDA_DEVICE ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost;
        NB_TRY(cudaMemcpyAsync(req->dst_rgba8, c->inference_rgba, bytes, kind, c->stream));
    }
    NB_TRY(cudaStreamSynchronize(c->stream));
    if (info) {
        info->capacity_bytes = bytes;
        info->valid_bytes = bytes;
        info->row_stride_bytes = c->width * 4u;
        info->width = c->width;
        info->height = c->height;
        info->generation = c->host_generation;
    }
    return NERF_STATUS_OK;
}

NERF_API NerfStatus nerf_save_network_weights(void* context, const NerfCheckpointFileDesc* desc) {
    if (!context || !desc || !desc->path_utf8) return NERF_STATUS_INVALID_USAGE;
    Context* c = as_ctx(context);
    std::lock_guard<std::mutex> lk(c->mu);
    std::vector<float> host(c->n_params);
    NB_TRY(cudaStreamSynchronize(c->stream));
    NB_TRY(c->read_sharded(host.data(), c->master, c->n_params));
    const auto tensors = nb::ckpt::layout(c->n_grid);
    std::string h = "{\"__metadata__\":{\"format\":\"nerf-b200/network-v1\"";
    char buf[512];
    std::snprintf(buf, sizeof(buf),
                  ",\"hash_levels\":%u,\"hash_features\":2,\"log2_hashmap_size\":%u,\"base_resolution\":%u,"
                  "\"max_resolution\":%u,\"density_input_dim\":32,\"density_hidden_layers\":1,\"density_width\":64,"
                  "\"density_output_dim\":16,\"color_input_dim\":32,\"color_hidden_layers\":2,\"color_width\":64,"
                  "\"color_output_dim\":16}",
                  c->grid.n_levels, c->grid.log2_hashmap_size, c->grid.base_resolution, c->grid.max_resolution);
    h += buf;
    uint64_t off = 0;
    for (const auto& t : tensors) {
        const uint64_t bytes = static_cast<uint64_t>(t.rows) * t.cols * 4u;
        std::snprintf(buf, sizeof(buf), ",\"%s\":{\"dtype\":\"F32\",\"shape\":[%u,%u],\"data_offsets\":[%llu,%llu]}",
                      t.name.c_str(), t.rows, t.cols, static_cast<unsigned long long>(off),
                      static_cast<unsigned long long>(off + bytes));
        h += buf;
        off += bytes;
    }
    h += "}";
    std::ofstream f(desc->path_utf8, std::ios::binary | std::ios::trunc);
    if (!f) return NERF_STATUS_IO_ERROR;
    const uint64_t len = h.size();
    f.write(reinterpret_cast<const char*>(&len), 8);
    f.write(h.data(), static_cast<std::streamsize>(h.size()));
    for (const auto& t : tensors)
        f.write(reinterpret_cast<const char*>(host.data() + t.offset), static_cast<std::streamsize>(uint64_t(t.rows) * t.cols * 4u));
    return f.good() ? NERF_STATUS_OK : NERF_STATUS_IO_ERROR;
}

NERF_API NerfStatus nerf_load_network_weights(void* context, const NerfCheckpointFileDesc* desc) {
    if (!context || !desc || !desc->path_utf8) return NERF_STATUS_INVALID_USAGE;
    Context* c = as_ctx(context);
    std::vector<float> host(c->n_params);
    try {
        std::ifstream f(desc->path_utf8, std::ios::binary);
        if (!f) return NERF_STATUS_IO_ERROR;
        uint64_t len = 0;
        f.read(reinterpret_cast<char*>(&len), 8);
        if (!f || len == 0u || len > (64ull << 20)) return NERF_STATUS_IO_ERROR;
        std::string header(len, '\0');
        f.read(header.data(), static_cast<std::streamsize>(len));
        if (!f) return NERF_STATUS_IO_ERROR;
        std::map<std::string, nb::ckpt::Entry> entries;
        if (!nb::ckpt::parse(header, entries)) return NERF_STATUS_IO_ERROR;
        for (const auto& t : nb::ckpt::layout(c->n_grid)) {
            auto it = entries.find(t.name);
            if (it == entries.end()) return NERF_STATUS_IO_ERROR;
            const auto& e = it->second;
            if (e.shape.size() != 2 || e.shape[0] != t.rows || e.shape[1] != t.cols || e.offsets.size() != 2) return NERF_STATUS_IO_ERROR;
            const uint64_t bytes = static_cast<uint64_t>(t.rows) * t.cols * 4u;
            if (e.offsets[1] - e.offsets[0] != bytes) return NERF_STATUS_IO_ERROR;
            f.seekg(static_cast<std::streamoff>(8u + len + e.offsets[0]), std::ios::beg);
            f.read(reinterpret_cast<char*>(host.data() + t.offset), static_cast<std::streamsize>(bytes));
            if (!f) return NERF_STATUS_IO_ERROR;
        }
    } catch (...) {
        return NERF_STATUS_IO_ERROR;
    }
    std::lock_guard<std::mutex> lk(c->mu);
    // Load resets optimiser, step and occupancy (reference backend-cuda.cu:2570-2591).
    NB_TRY(cudaStreamSynchronize(c->stream));
    NB_TRY(cudaMemcpy(c->master, host.data(), c->n_params * 4, cudaMemcpyHostToDevice));
    NB_TRY(nb::launch_f32_to_f16(c->master, c->p16, c->n_params, c->stream));
    NB_TRY(cudaMemsetAsync(c->m, 0, c->n_params * 4, c->stream));
    NB_TRY(cudaMemsetAsync(c->v, 0, c->n_params * 4, c->stream));
    NB_TRY(cudaMemsetAsync(c->grid_grad, 0, c->n_grid * 2, c->stream));
    NB_TRY(cudaMemsetAsync(c->mlp_grad, 0, nb::kMlpGradSlots * 4, c->stream));
    nb::DeviceState st{};
    st.n_rays = c->configured ? c->cfg.rays_per_batch : 0u;
    NB_TRY(cudaMemcpyAsync(c->state, &st, sizeof(st), cudaMemcpyHostToDevice, c->stream));
    c->stats_host_current = false;
    NB_TRY(cudaMemsetAsync(c->density, 0, static_cast<uint64_t>(c->words) * 32u * 4u, c->stream));
    NB_TRY(cudaMemsetAsync(c->bitfield, 0, c->words * 4ull, c->stream));
    if (c->configured) NB_TRY(nb::launch_march(c->sampler_args(), c->stream));  // the step state restarted at frame 0
    NB_TRY(cudaStreamSynchronize(c->stream));
    c->occupancy_valid = false;
    c->host_generation = 0;
    return NERF_STATUS_OK;
}

// Training-state checkpoint: the same container (u64 header length, JSON
// header, raw tensors) with every tensor a training step reads besides the
// dataset: fp32 masters, both Adam moments, the occupancy densities and
// bitfield, and the step state (frame, ray count, counters, last statistics).
namespace {
struct StateBlob {
    const char* name;
    const char* dtype;
    uint64_t count, elem;
    void* host;
};
std::vector<StateBlob> state_blobs(Context* c, std::vector<float>& master, std::vector<float>& am, std::vector<float>& av,
                                   std::vector<float>& density, std::vector<uint32_t>& bits, nb::DeviceState& st) {
    master.resize(c->n_params);
    am.resize(c->n_params);
    av.resize(c->n_params);
    density.resize(c->cell_count);
    bits.resize(c->words);
    return {{"params.master", "F32", c->n_params, 4u, master.data()},
            {"adam.m", "F32", c->n_params, 4u, am.data()},
            {"adam.v", "F32", c->n_params, 4u, av.data()},
            {"occupancy.density", "F32", c->cell_count, 4u, density.data()},
            {"occupancy.bitfield", "U32", c->words, 4u, bits.data()},
            {"step.state", "U8", sizeof(nb::DeviceState), 1u, &st}};
}
}  // namespace

NERF_API NerfStatus nerf_b200_save_training_state(void* context, const char* path_utf8) {
    if (!context || !path_utf8) return NERF_STATUS_INVALID_USAGE;
    Context* c = as_ctx(context);
    std::lock_guard<std::mutex> lk(c->mu);
    if (!c->configured) return NERF_STATUS_STATE_ERROR;
    std::vector<float> master, am, av, density;
    std::vector<uint32_t> bits;
    nb::DeviceState st{};
    const auto blobs = state_blobs(c, master, am, av, density, bits, st);
    NB_TRY(cudaStreamSynchronize(c->stream));
    NB_TRY(c->read_sharded(master.data(), c->master, c->n_params));
    NB_TRY(c->read_sharded(am.data(), c->m, c->n_params));
    NB_TRY(c->read_sharded(av.data(), c->v, c->n_params));
    NB_TRY(cudaMemcpy(density.data(), c->density, c->cell_count * 4ull, cudaMemcpyDeviceToHost));
    NB_TRY(cudaMemcpy(bits.data(), c->bitfield, c->words * 4ull, cudaMemcpyDeviceToHost));
    NB_TRY(cudaMemcpy(&st, c->state, sizeof(st), cudaMemcpyDeviceToHost));
    char buf[512];
    std::snprintf(buf, sizeof(buf),
                  "{\"__metadata__\":{\"format\":\"nerf-b200/training-state-v1\",\"log2_hashmap_size\":%u,"
                  "\"base_resolution\":%u,\"max_resolution\":%u,\"occupancy_grid_res\":%u,\"frame_index\":%u}",
                  c->grid.log2_hashmap_size, c->grid.base_resolution, c->grid.max_resolution, c->grid_res, st.frame_index);
    std::string h = buf;
    uint64_t off = 0;
    for (const auto& b : blobs) {
        std::snprintf(buf, sizeof(buf), ",\"%s\":{\"dtype\":\"%s\",\"shape\":[%llu],\"data_offsets\":[%llu,%llu]}", b.name,
                      b.dtype, static_cast<unsigned long long>(b.count), static_cast<unsigned long long>(off),
                      static_cast<unsigned long long>(off + b.count * b.elem));
        h += buf;
        off += b.count * b.elem;
    }
    h += "}";
    std::ofstream f(path_utf8, std::ios::binary | std::ios::trunc);
    if (!f) return NERF_STATUS_IO_ERROR;
    const uint64_t len = h.size();
    f.write(reinterpret_cast<const char*>(&len), 8);
    f.write(h.data(), static_cast<std::streamsize>(h.size()));
    for (const auto& b : blobs) f.write(static_cast<const char*>(b.host), static_cast<std::streamsize>(b.count * b.elem));
    return f.good() ? NERF_STATUS_OK : NERF_STATUS_IO_ERROR;
}

NERF_API NerfStatus nerf_b200_load_training_state(void* context, const char* path_utf8) {
    if (!context || !path_utf8) return NERF_STATUS_INVALID_USAGE;
    Context* c = as_ctx(context);
    if (!c->configured) return NERF_STATUS_STATE_ERROR;
    std::vector<float> master, am, av, density;
    std::vector<uint32_t> bits;
    nb::DeviceState st{};
    const auto blobs = state_blobs(c, master, am, av, density, bits, st);
    try {
        std::ifstream f(path_utf8, std::ios::binary);
        if (!f) return NERF_STATUS_IO_ERROR;
        uint64_t len = 0;
        f.read(reinterpret_cast<char*>(&len), 8);
        if (!f || len == 0u || len > (64ull << 20)) return NERF_STATUS_IO_ERROR;
        std::string header(len, '\0');
        f.read(header.data(), static_cast<std::streamsize>(len));
        if (!f) return NERF_STATUS_IO_ERROR;
        std::map<std::string, nb::ckpt::Entry> entries;
        if (!nb::ckpt::parse(header, entries)) return NERF_STATUS_IO_ERROR;
        for (const auto& b : blobs) {  // every tensor present with this context's size
            auto it = entries.find(b.name);
            if (it == entries.end()) return NERF_STATUS_IO_ERROR;
            const auto& e = it->second;
            if (e.shape.size() != 1 || e.shape[0] != b.count || e.offsets.size() != 2 || e.offsets[1] - e.offsets[0] != b.count * b.elem)
                return NERF_STATUS_IO_ERROR;
            f.seekg(static_cast<std::streamoff>(8u + len + e.offsets[0]), std::ios::beg);
            f.read(static_cast<char*>(b.host), static_cast<std::streamsize>(b.count * b.elem));
            if (!f) return NERF_STATUS_IO_ERROR;
        }
    } catch (...) {
        return NERF_STATUS_IO_ERROR;
    }
    std::lock_guard<std::mutex> lk(c->mu);
    NB_TRY(cudaStreamSynchronize(c->stream));
    // Every rank writes the whole vectors (peer mode reads only its owned range).
    NB_TRY(cudaMemcpy(c->master, master.data(), c->n_params * 4, cudaMemcpyHostToDevice));
    NB_TRY(cudaMemcpy(c->m, am.data(), c->n_params * 4, cudaMemcpyHostToDevice));
    NB_TRY(cudaMemcpy(c->v, av.data(), c->n_params * 4, cudaMemcpyHostToDevice));
    NB_TRY(nb::launch_f32_to_f16(c->master, c->p16, c->n_params, c->stream));  // the fp16 mirror is rn(master)
    NB_TRY(cudaMemsetAsync(c->grid_grad, 0, c->n_grid * 2, c->stream));
    NB_TRY(cudaMemsetAsync(c->mlp_grad, 0, nb::kMlpGradSlots * 4, c->stream));
    NB_TRY(cudaMemcpyAsync(c->density, density.data(), c->cell_count * 4ull, cudaMemcpyHostToDevice, c->stream));
    NB_TRY(cudaMemcpyAsync(c->bitfield, bits.data(), c->words * 4ull, cudaMemcpyHostToDevice, c->stream));
    st.done_blocks = 0u;
    st.grad_sumsq = 0.0f;
    st.nonfinite = 0u;
    NB_TRY(cudaMemcpyAsync(c->state, &st, sizeof(st), cudaMemcpyHostToDevice, c->stream));
    c->stats_host_current = false;
    NB_TRY(nb::launch_march(c->sampler_args(), c->stream));  // the next step's march (frame and ray count restored)
    NB_TRY(cudaStreamSynchronize(c->stream));
    c->occupancy_valid = true;
    c->host_generation = st.frame_index;
    return NERF_STATUS_OK;
}

// ============================================================= nerf_b200.h
NERF_API NerfStatus nerf_b200_read_counters(void* context, NerfB200Counters* out) {
    if (!context || !out) return NERF_STATUS_INVALID_USAGE;
    Context* c = as_ctx(context);
    std::lock_guard<std::mutex> lk(c->mu);
    nb::DeviceState st{};
    NB_TRY(cudaMemcpyAsync(&st, c->state, sizeof(st), cudaMemcpyDeviceToHost, c->stream));
    NB_TRY(cudaStreamSynchronize(c->stream));
    out->frame_index = st.frame_index;
    out->rays = st.last_rays;
    out->active_rays = st.last_active;
    out->samples = st.last_samples;
    out->marched_active_rays = st.n_marched_active;
    out->next_rays = st.n_rays;
    out->total_samples = st.total_samples;
    out->total_rays = st.total_rays;
    // occupancy query + update, sampler (3), forward, composite, backward MLP +
    // scatter, statistics, march, Adam; data-parallel: + weight-gradient
    // reduce, and in peer mode 3 barriers + the gradient reduction.
    // occupancy query + update, march, 3 sampler kernels, forward, composite,
    // MLP backward + scatter, statistics, Adam (the tensor-core path splits the
    // forward into encode + MLP); data parallel adds the weight-gradient
    // reduction, and peer mode its barriers and gradient reduction.
    out->kernels_per_step = 12u + (c->mlp_tc ? 1u : 0u) + (c->dp_active() ? 1u : 0u) + (c->dp_peer ? 4u : 0u);
    out->dp_peer = c->dp_peer ? 1u : 0u;
    return NERF_STATUS_OK;
}

NERF_API NerfStatus nerf_b200_grid_layout(uint32_t L, uint32_t log2T, uint32_t base, uint32_t maxres, NerfB200GridLayout* out) {
    if (!out) return NERF_STATUS_INVALID_USAGE;
    return nb::grid_layout(L, log2T, base, maxres, reinterpret_cast<nb::GridLayout*>(out)) == 0 ? NERF_STATUS_OK
                                                                                              : NERF_STATUS_INVALID_USAGE;
}

NERF_API NerfStatus nerf_b200_context_grid_layout(void* context, NerfB200GridLayout* out) {
    if (!context || !out) return NERF_STATUS_INVALID_USAGE;
    std::memcpy(out, &as_ctx(context)->grid, sizeof(*out));
    return NERF_STATUS_OK;
}

NERF_API NerfStatus nerf_b200_param_counts(void* context, uint64_t* n_grid, uint64_t* n_mlp) {
    if (!context) return NERF_STATUS_INVALID_USAGE;
    if (n_grid) *n_grid = as_ctx(context)->n_grid;
    if (n_mlp) *n_mlp = nb::kMlpParams;
    return NERF_STATUS_OK;
}

NERF_API NerfStatus nerf_b200_read_params(void* context, float* master, uint16_t* p16, float* am, float* av) {
    if (!context) return NERF_STATUS_INVALID_USAGE;
    Context* c = as_ctx(context);
    std::lock_guard<std::mutex> lk(c->mu);
    NB_TRY(cudaStreamSynchronize(c->stream));
    const uint64_t n = c->n_params;
    if (master) NB_TRY(c->read_sharded(master, c->master, n));
    if (p16) NB_TRY(cudaMemcpy(p16, c->p16, n * 2, cudaMemcpyDeviceToHost));
    if (am) NB_TRY(c->read_sharded(am, c->m, n));
    if (av) NB_TRY(c->read_sharded(av, c->v, n));
    return NERF_STATUS_OK;
}

NERF_API NerfStatus nerf_b200_write_params(void* context, const float* master) {
    if (!context || !master) return NERF_STATUS_INVALID_USAGE;
    Context* c = as_ctx(context);
    std::lock_guard<std::mutex> lk(c->mu);
    NB_TRY(cudaStreamSynchronize(c->stream));
    NB_TRY(cudaMemcpy(c->master, master, c->n_params * 4, cudaMemcpyHostToDevice));
    NB_TRY(nb::launch_f32_to_f16(c->master, c->p16, c->n_params, c->stream));
    NB_TRY(cudaStreamSynchronize(c->stream));
    return NERF_STATUS_OK;
}

NERF_API NerfStatus nerf_b200_read_occupancy(void* context, float* density, uint32_t* bitfield) {
    if (!context) return NERF_STATUS_INVALID_USAGE;
    Context* c = as_ctx(context);
    std::lock_guard<std::mutex> lk(c->mu);
    NB_TRY(cudaStreamSynchronize(c->stream));
    if (density) NB_TRY(cudaMemcpy(density, c->density, c->cell_count * 4ull, cudaMemcpyDeviceToHost));
    if (bitfield) NB_TRY(cudaMemcpy(bitfield, c->bitfield, c->words * 4ull, cudaMemcpyDeviceToHost));
    return NERF_STATUS_OK;
}

NERF_API NerfStatus nerf_b200_write_occupancy(void* context, const float* density, const uint32_t* bitfield) {
    if (!context) return NERF_STATUS_INVALID_USAGE;
    Context* c = as_ctx(context);
    std::lock_guard<std::mutex> lk(c->mu);
    NB_TRY(cudaStreamSynchronize(c->stream));
    if (density) NB_TRY(cudaMemcpy(c->density, density, c->cell_count * 4ull, cudaMemcpyHostToDevice));
    if (bitfield) {
        NB_TRY(cudaMemcpy(c->bitfield, bitfield, c->words * 4ull, cudaMemcpyHostToDevice));
        c->occupancy_valid = true;
    }
    return NERF_STATUS_OK;
}

NERF_API NerfStatus nerf_b200_set_frame_index(void* context, uint32_t frame) {
    if (!context) return NERF_STATUS_INVALID_USAGE;
    Context* c = as_ctx(context);
    std::lock_guard<std::mutex> lk(c->mu);
    NB_TRY(cudaMemcpyAsync(&c->state->frame_index, &frame, 4, cudaMemcpyHostToDevice, c->stream));
    if (c->configured) NB_TRY(nb::launch_march(c->sampler_args(), c->stream));  // the march depends on the frame
    NB_TRY(cudaStreamSynchronize(c->stream));
    return NERF_STATUS_OK;
}

NERF_API NerfStatus nerf_b200_read_batch(void* context, uint32_t* ray_counts, uint32_t* ray_index, NerfB200RayRecord* recs,
                                         float* pos_dt, uint32_t* sample_ray) {
    if (!context) return NERF_STATUS_INVALID_USAGE;
    Context* c = as_ctx(context);
    std::lock_guard<std::mutex> lk(c->mu);
    if (!c->configured) return NERF_STATUS_STATE_ERROR;
    nb::DeviceState st{};
    NB_TRY(cudaMemcpyAsync(&st, c->state, sizeof(st), cudaMemcpyDeviceToHost, c->stream));
    NB_TRY(cudaStreamSynchronize(c->stream));
    if (ray_counts)
        NB_TRY(cudaMemcpy(ray_counts, c->ray_counts + static_cast<uint64_t>(st.counts_parity) * c->tc.max_rays,
                          st.last_rays * 4ull, cudaMemcpyDeviceToHost));
    if (ray_index) NB_TRY(cudaMemcpy(ray_index, c->ray_index, st.last_active * 4ull, cudaMemcpyDeviceToHost));
    if (recs) NB_TRY(cudaMemcpy(recs, c->rays, st.last_active * sizeof(nb::RayRecord), cudaMemcpyDeviceToHost));
    if (pos_dt) NB_TRY(cudaMemcpy(pos_dt, c->pos_dt, st.last_samples * 16ull, cudaMemcpyDeviceToHost));
    if (sample_ray) NB_TRY(cudaMemcpy(sample_ray, c->sample_ray, st.last_samples * 4ull, cudaMemcpyDeviceToHost));
    return NERF_STATUS_OK;
}

NERF_API NerfStatus nerf_b200_dp_unique_id(uint8_t out[NERF_B200_DP_ID_BYTES]) {
    if (!out) return NERF_STATUS_INVALID_USAGE;
    std::lock_guard<std::mutex> lk(nb::g_nccl_mu);
    if (!nb::g_nccl.load()) return NERF_STATUS_FAILURE;
    ncclUniqueId id;
    static_assert(sizeof(id) == NERF_B200_DP_ID_BYTES, "nccl id size");
    if (nb::g_nccl.get_unique_id(&id) != ncclSuccess) return NERF_STATUS_FAILURE;
    std::memcpy(out, &id, sizeof(id));
    return NERF_STATUS_OK;
}

NERF_API NerfStatus nerf_b200_dp_init(void* context, uint32_t rank, uint32_t world, const uint8_t id[NERF_B200_DP_ID_BYTES]) {
    if (!context || !id || world == 0u || rank >= world) return NERF_STATUS_INVALID_USAGE;
    Context* c = as_ctx(context);
    std::lock_guard<std::mutex> lk(c->mu);
    if (c->comm) return NERF_STATUS_STATE_ERROR;
    c->dp_rank = rank;
    c->dp_world = world;
    if (const char* t = std::getenv("NERF_B200_DP_TIMEOUT_MS")) {
        const double ms = std::atof(t);
        if (ms > 0.0) c->dp_timeout_ns = static_cast<uint64_t>(ms * 1e6);
    }
    if (world == 1u) return NERF_STATUS_OK;
    {
        std::lock_guard<std::mutex> lk2(nb::g_nccl_mu);
        if (!nb::g_nccl.load()) return NERF_STATUS_FAILURE;
    }
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    if (nb::g_nccl.comm_init_rank(&c->comm, static_cast<int>(world), uid, static_cast<int>(rank)) != ncclSuccess) {
        c->comm = nullptr;
        return NERF_STATUS_FAILURE;
    }
    const NerfStatus ps = c->open_peers();
    if (ps != NERF_STATUS_OK) return ps;
    c->configured = false;  // the step graph must be recaptured with the exchange
    return NERF_STATUS_OK;
}

NERF_API NerfStatus nerf_b200_dp_peer_handle(void* context, uint8_t out[NERF_B200_DP_HANDLE_BYTES]) {
    if (!context || !out) return NERF_STATUS_INVALID_USAGE;
    Context* c = as_ctx(context);
    std::lock_guard<std::mutex> lk(c->mu);
    cudaIpcMemHandle_t h{};
    if (cudaIpcGetMemHandle(&h, c->model.base) != cudaSuccess) {
        cudaGetLastError();
        return NERF_STATUS_CUDA_ERROR;
    }
    std::memset(out, 0, NERF_B200_DP_HANDLE_BYTES);
    std::memcpy(out, &h, sizeof(h));
    const uint64_t meta[2] = {c->model.size, c->n_params};
    std::memcpy(out + sizeof(h), meta, sizeof(meta));
    std::memcpy(out + sizeof(h) + sizeof(meta), &nb::kDpHandleMagic, 4);
    return NERF_STATUS_OK;
}

NERF_API NerfStatus nerf_b200_dp_init_peers(void* context, uint32_t rank, uint32_t world, const uint8_t* handles) {
    static_assert(sizeof(cudaIpcMemHandle_t) + 20 <= NERF_B200_DP_HANDLE_BYTES, "handle layout");
    if (!context || !handles || world < 2u || world > nb::kMaxDpWorld || rank >= world) return NERF_STATUS_INVALID_USAGE;
    Context* c = as_ctx(context);
    std::lock_guard<std::mutex> lk(c->mu);
    if (c->comm || c->dp_peer || c->dp_world != 1u) return NERF_STATUS_STATE_ERROR;
    const size_t hb = sizeof(cudaIpcMemHandle_t);
    for (uint32_t r = 0; r < world; ++r) {  // every rank's arena has this rank's layout
        const uint8_t* h = handles + static_cast<size_t>(NERF_B200_DP_HANDLE_BYTES) * r;
        uint64_t meta[2];
        uint32_t magic = 0;
        std::memcpy(meta, h + hb, sizeof(meta));
        std::memcpy(&magic, h + hb + sizeof(meta), 4);
        if (magic != nb::kDpHandleMagic || meta[0] != c->model.size || meta[1] != c->n_params) return NERF_STATUS_INVALID_USAGE;
    }
    if (const char* t = std::getenv("NERF_B200_DP_TIMEOUT_MS")) {
        const double ms = std::atof(t);
        if (ms > 0.0) c->dp_timeout_ns = static_cast<uint64_t>(ms * 1e6);
    }
    c->dp_rank = rank;
    c->dp_world = world;
    if (!c->map_peers(handles)) {
        c->dp_rank = 0u;
        c->dp_world = 1u;
        return NERF_STATUS_FAILURE;
    }
    c->dp_peer = true;
    c->configured = false;  // the step graph must be recaptured with the exchange
    return NERF_STATUS_OK;
}

NERF_API NerfStatus nerf_b200_dp_barrier_test(void* context, uint32_t timeout_us) {
    if (!context || timeout_us == 0u) return NERF_STATUS_INVALID_USAGE;
    Context* c = as_ctx(context);
    std::lock_guard<std::mutex> lk(c->mu);
    if (!c->configured) return NERF_STATUS_STATE_ERROR;
    if (c->dp_active()) return NERF_STATUS_STATE_ERROR;  // only on a context that trains alone
    if (!c->dp_absent) {
        if (cudaMalloc(&c->dp_absent, sizeof(nb::DpSync)) != cudaSuccess) {
            c->dp_absent = nullptr;
            return NERF_STATUS_FAILURE;
        }
        NB_TRY(cudaMemsetAsync(c->dp_absent, 0, sizeof(nb::DpSync), c->stream));
    }
    nb::DpPeers d{};
    d.world = 2u;
    d.rank = 0u;
    d.sync[0] = c->dp_sync;
    d.sync[1] = c->dp_absent;  // rank 1 never announces an epoch
    d.timeout_ns = static_cast<uint64_t>(timeout_us) * 1000u;
    c->dp_watch = true;
    return nb::cuda_status(nb::launch_dp_barrier(d, c->stream));
}

NERF_API NerfStatus nerf_b200_render(void* context, const NerfB200RenderRequest* r, NerfB200RenderInfo* info) {
    if (!context || !r || !r->c2w_3x4) return NERF_STATUS_INVALID_USAGE;
    Context* c = as_ctx(context);
    std::lock_guard<std::mutex> lk(c->mu);
    const uint64_t bytes = static_cast<uint64_t>(r->width) * r->height * 4u;
    if (r->dst_rgba8 && r->dst_bytes < bytes) return NERF_STATUS_INVALID_USAGE;
    const float stop = r->stop_transmittance < 0.0f ? c->opt.render_stop_transmittance : r->stop_transmittance;
    const NerfStatus s = c->render_view(r->c2w_3x4, r->width, r->height, r->fx, r->fy, r->cx, r->cy, r->max_steps, stop,
                                        r->tile_size, r->tile_rank, r->tile_world, info);
    if (s != NERF_STATUS_OK) return s;
    if (r->dst_rgba8) {
        const cudaMemcpyKind kind = r->memory_kind == NERF_MEMORY_CUDA_DEVICE ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost;
        NB_TRY(cudaMemcpyAsync(r->dst_rgba8, c->render_rgba, bytes, kind, c->stream));
    }
    NB_TRY(cudaStreamSynchronize(c->stream));
    return NERF_STATUS_OK;
}

NERF_API NerfStatus nerf_b200_render_output(void* context, const void** device_rgba8) {
    if (!context || !device_rgba8) return NERF_STATUS_INVALID_USAGE;
    *device_rgba8 = as_ctx(context)->render_rgba;
    return NERF_STATUS_OK;
}

NERF_API NerfStatus nerf_b200_context_stream(void* context, void** stream) {
    if (!context || !stream) return NERF_STATUS_INVALID_USAGE;
    *stream = as_ctx(context)->stream;
    return NERF_STATUS_OK;
}

NERF_API NerfStatus nerf_b200_train_step_profiled(void* context, NerfB200StepProfile* out) {
    if (!context || !out) return NERF_STATUS_INVALID_USAGE;
    Context* c = as_ctx(context);
    std::lock_guard<std::mutex> lk(c->mu);
    if (!c->configured) return NERF_STATUS_STATE_ERROR;
    cudaEvent_t ev[nb::kStepKernels + 1] = {};
    NerfStatus st = NERF_STATUS_OK;
    for (auto& e : ev)
        if (cudaEventCreate(&e) != cudaSuccess) st = NERF_STATUS_CUDA_ERROR;
    if (st == NERF_STATUS_OK && c->enqueue_step(c->stream, ev) != cudaSuccess) st = NERF_STATUS_CUDA_ERROR;
    if (st == NERF_STATUS_OK) c->stats_host_current = true;
    if (st == NERF_STATUS_OK && cudaStreamSynchronize(c->stream) != cudaSuccess) st = NERF_STATUS_CUDA_ERROR;
    if (st == NERF_STATUS_OK) {
        for (int k = 0; k < nb::kStepKernels; ++k) cudaEventElapsedTime(&out->milliseconds[k], ev[k], ev[k + 1]);
        cudaEventElapsedTime(&out->total_milliseconds, ev[0], ev[nb::kStepKernels]);
        ++c->host_generation;
        c->occupancy_valid = true;
    }
    for (auto& e : ev)
        if (e) cudaEventDestroy(e);
    return st;
}

// ------------------------------------------------------ kernel-level entries
// Parameter and gradient tables of the kernel-level entry points are read
// and reduced in 16-byte blocks.
static bool misaligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) != 0u; }

NERF_API NerfStatus nerf_b200_grid_forward(const NerfB200GridLayout* layout, const float* pos, uint32_t n, const void* params,
                                           void* feat, void* stream) {
    if (!layout || (n && (!pos || !params || !feat))) return NERF_STATUS_INVALID_USAGE;
    if (misaligned16(params)) return NERF_STATUS_INVALID_USAGE;
    const nb::LevelTable lt = nb::make_level_table(*reinterpret_cast<const nb::GridLayout*>(layout));
    return nb::cuda_status(nb::launch_grid_forward(lt, pos, n, params, feat, static_cast<cudaStream_t>(stream)));
}

NERF_API NerfStatus nerf_b200_grid_backward(const NerfB200GridLayout* layout, const float* pos, uint32_t n, const void* dfeat,
                                            void* grad, void* stream) {
    if (!layout || (n && (!pos || !dfeat || !grad))) return NERF_STATUS_INVALID_USAGE;
    if (misaligned16(grad)) return NERF_STATUS_INVALID_USAGE;
    const nb::LevelTable lt = nb::make_level_table(*reinterpret_cast<const nb::GridLayout*>(layout));
    return nb::cuda_status(nb::launch_grid_backward(lt, pos, n, dfeat, grad, static_cast<cudaStream_t>(stream)));
}

NERF_API NerfStatus nerf_b200_field_forward(const NerfB200GridLayout* layout, const void* params, const float* pos,
                                            const float* dirs, uint32_t n, void* feat, float* raw, void* stream) {
    if (!layout || layout->n_levels != 16u || (n && (!params || !pos || !dirs || !raw))) return NERF_STATUS_INVALID_USAGE;
    if (misaligned16(params)) return NERF_STATUS_INVALID_USAGE;
    if (nb::ensure_attributes() != cudaSuccess) return NERF_STATUS_CUDA_ERROR;
    nb::FieldArgs a{};
    a.lt = nb::make_level_table(*reinterpret_cast<const nb::GridLayout*>(layout));
    a.params16 = params;
    a.mlp_offset = 2u * layout->offset[layout->n_levels];
    a.n_direct = n;
    a.pos_unit = pos;
    a.dirs = dirs;
    a.feat = feat;
    a.raw = reinterpret_cast<float4*>(raw);
    if (n == 0u) return NERF_STATUS_OK;
    return nb::cuda_status(nb::launch_field_forward(a, nb::kFieldDirect, nb::field_forward_blocks(), static_cast<cudaStream_t>(stream)));
}

NERF_API uint64_t nerf_b200_field_backward_partial_floats(void) {
    if (nb::ensure_attributes() != cudaSuccess) return 0u;
    return static_cast<uint64_t>(nb::field_backward_blocks()) * nb::kMlpParams;
}

NERF_API NerfStatus nerf_b200_field_backward(const NerfB200GridLayout* layout, const void* params, const float* pos,
                                             const float* dirs, uint32_t n, const void* feat, const float* dout,
                                             void* grid_grad, float* partials, float* mlp_grad, void* stream) {
    if (!layout || layout->n_levels != 16u || !params || !partials || !mlp_grad || !grid_grad) return NERF_STATUS_INVALID_USAGE;
    if (misaligned16(params) || misaligned16(grid_grad)) return NERF_STATUS_INVALID_USAGE;
    if (n && (!pos || !dirs || !feat || !dout)) return NERF_STATUS_INVALID_USAGE;
    if (n > 0x7FFFFFFFu) return NERF_STATUS_INVALID_USAGE;  // rows are indexed with 32-bit tile counters
    if (nb::ensure_attributes() != cudaSuccess) return NERF_STATUS_CUDA_ERROR;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    nb::FieldArgs a{};
    a.lt = nb::make_level_table(*reinterpret_cast<const nb::GridLayout*>(layout));
    a.params16 = params;
    a.mlp_offset = 2u * layout->offset[layout->n_levels];
    a.n_direct = n;
    a.pos_unit = pos;
    a.dirs = dirs;
    a.feat = const_cast<void*>(feat);
    a.dout = reinterpret_cast<const float4*>(dout);
    a.grid_grad = grid_grad;
    a.partials = partials;
    const uint32_t blocks = nb::field_backward_blocks();
    cudaError_t e = nb::launch_field_backward(a, nb::kFieldDirect, blocks, s);
    if (e != cudaSuccess) return NERF_STATUS_CUDA_ERROR;
    nb::OptimArgs o{};
    o.partials = partials;
    o.n_partials = blocks;
    o.mlp_grad = mlp_grad;
    return nb::cuda_status(nb::launch_wgrad_reduce(o, s));
}

NERF_API NerfStatus nerf_b200_mlp_forward(const void* mlp_params, const void* feat, const float* dirs, uint32_t n, float* raw,
                                          void* stream) {
    if (n && (!mlp_params || !feat || !dirs || !raw)) return NERF_STATUS_INVALID_USAGE;
    if (misaligned16(mlp_params)) return NERF_STATUS_INVALID_USAGE;
    if (n == 0u) return NERF_STATUS_OK;
    if (nb::ensure_attributes() != cudaSuccess) return NERF_STATUS_CUDA_ERROR;
    nb::FieldArgs a{};
    a.params16 = mlp_params;
    a.mlp_offset = 0u;
    a.n_direct = n;
    a.dirs = dirs;
    a.feat = const_cast<void*>(feat);
    a.raw = reinterpret_cast<float4*>(raw);
    return nb::cuda_status(nb::launch_field_forward(a, nb::kFieldMlp, nb::field_forward_blocks(), static_cast<cudaStream_t>(stream)));
}

NERF_API NerfStatus nerf_b200_mlp_forward_tc(const void* mlp_params, const void* feat, const float* dirs, uint32_t n, float* raw,
                                             uint32_t* error_word, void* stream) {
    if (n && (!mlp_params || !feat || !dirs || !raw || !error_word)) return NERF_STATUS_INVALID_USAGE;
    if (misaligned16(mlp_params)) return NERF_STATUS_INVALID_USAGE;
    if (n == 0u) return NERF_STATUS_OK;
    return nb::cuda_status(nb::launch_mlp_forward_tc(mlp_params, feat, dirs, n, raw, error_word, static_cast<cudaStream_t>(stream)));
}

NERF_API NerfStatus nerf_b200_mlp_tc_info(uint32_t out[4]) {
    if (!out) return NERF_STATUS_INVALID_USAGE;
    nb::mlp_tc_info(out);
    return out[0] ? NERF_STATUS_OK : NERF_STATUS_CUDA_ERROR;
}

NERF_API NerfStatus nerf_b200_mlp_backward_tc(const void* mlp_params, const void* feat, const float* dirs, uint32_t n,
                                              const float* dout, void* dfeat, float* partials, float* mlp_grad, uint32_t* error_word,
                                              void* stream) {
    if (!mlp_params || !partials || !mlp_grad || !error_word) return NERF_STATUS_INVALID_USAGE;
    if (misaligned16(mlp_params)) return NERF_STATUS_INVALID_USAGE;
    if (n && (!feat || !dirs || !dout || !dfeat)) return NERF_STATUS_INVALID_USAGE;
    if (nb::ensure_attributes() != cudaSuccess) return NERF_STATUS_CUDA_ERROR;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const uint32_t cap = nb::mlp_backward_tc_blocks();
    if (cap == 0u || cap > nb::field_backward_blocks()) return NERF_STATUS_CUDA_ERROR;  // partials sized for the field backward
    const uint32_t tiles = (n + 127u) / 128u;
    const uint32_t blocks = tiles == 0u ? 1u : (tiles < cap ? tiles : cap);
    if (nb::launch_mlp_backward_tc(mlp_params, feat, 0, dirs, dout, nullptr, n, dfeat, partials, blocks, error_word, s) != cudaSuccess)
        return NERF_STATUS_CUDA_ERROR;
    nb::OptimArgs o{};
    o.partials = partials;
    o.n_partials = blocks;
    o.mlp_grad = mlp_grad;
    return nb::cuda_status(nb::launch_wgrad_reduce(o, s));
}

NERF_API NerfStatus nerf_b200_mlp_backward(const void* mlp_params, const void* feat, const float* dirs, uint32_t n,
                                           const float* dout, void* dfeat, float* partials, float* mlp_grad, void* stream) {
    if (!mlp_params || !partials || !mlp_grad) return NERF_STATUS_INVALID_USAGE;
    if (misaligned16(mlp_params)) return NERF_STATUS_INVALID_USAGE;
    if (n && (!feat || !dirs || !dout || !dfeat)) return NERF_STATUS_INVALID_USAGE;
    if (nb::ensure_attributes() != cudaSuccess) return NERF_STATUS_CUDA_ERROR;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    nb::FieldArgs a{};
    a.params16 = mlp_params;
    a.mlp_offset = 0u;
    a.n_direct = n;
    a.dirs = dirs;
    a.feat = const_cast<void*>(feat);
    a.dout = reinterpret_cast<const float4*>(dout);
    a.dfeat = dfeat;
    a.partials = partials;
    const uint32_t blocks = nb::field_backward_blocks();
    if (nb::launch_field_backward(a, nb::kFieldMlp, blocks, s) != cudaSuccess) return NERF_STATUS_CUDA_ERROR;
    nb::OptimArgs o{};
    o.partials = partials;
    o.n_partials = blocks;
    o.mlp_grad = mlp_grad;
    return nb::cuda_status(nb::launch_wgrad_reduce(o, s));
}

NERF_API NerfStatus nerf_b200_composite(const NerfB200RayRecord* rays, uint32_t n_rays, const float* raw, const float* pos_dt,
                                        float inv_norm, float loss_scale, float stop, float* dout, float* ray_loss,
                                        uint32_t* ray_used, float* loss_sum, void* stream) {
    if (n_rays && (!rays || !raw || !pos_dt || !dout)) return NERF_STATUS_INVALID_USAGE;
    nb::CompositeArgs a{};
    a.rays = reinterpret_cast<const nb::RayRecord*>(rays);
    a.raw = reinterpret_cast<const float4*>(raw);
    a.pos_dt = reinterpret_cast<const float4*>(pos_dt);
    a.dout = reinterpret_cast<float4*>(dout);
    a.loss_slot = loss_sum;
    a.loss_scale = loss_scale;
    a.stop_transmittance = stop;
    a.direct = 1;
    a.n_rays = n_rays;
    a.inv_norm = inv_norm;
    a.ray_loss = ray_loss;
    a.ray_used = ray_used;
    a.dp_world = 1;
    return nb::cuda_status(nb::launch_composite(a, static_cast<cudaStream_t>(stream)));
}

NERF_API NerfStatus nerf_b200_adam(float* master, void* p16, void* grid_grad, const float* mlp_grad, float* am, float* av,
                                   uint64_t n_grid, uint64_t n_params, const float scalars[5], uint32_t skip, float beta1,
                                   float beta2, float eps, void* stream) {
    if (!master || !p16 || !am || !av || !scalars || n_params < n_grid || (n_grid % 16u) || (n_params % 8u))
        return NERF_STATUS_INVALID_USAGE;
    if (n_grid && !grid_grad) return NERF_STATUS_INVALID_USAGE;
    if (n_params > n_grid && !mlp_grad) return NERF_STATUS_INVALID_USAGE;
    nb::OptimArgs o{};
    o.master = master;
    o.params16 = p16;
    o.grid_grad = grid_grad;
    o.mlp_grad = const_cast<float*>(mlp_grad);
    o.mlp_in = mlp_grad;
    o.m = am;
    o.v = av;
    o.n_grid = n_grid;
    o.n_params = n_params;
    o.tc.beta1 = beta1;
    o.tc.beta2 = beta2;
    o.tc.eps = eps;
    o.direct_scalars.learning_rate = scalars[0];
    o.direct_scalars.grad_scale = scalars[1];
    o.direct_scalars.inv_bias_correction1 = scalars[2];
    o.direct_scalars.inv_bias_correction2 = scalars[3];
    o.direct_scalars.inv_loss_scale = scalars[4];
    o.direct_scalars.skip_update = skip;
    return nb::cuda_status(nb::launch_adam(o, static_cast<cudaStream_t>(stream)));
}

NERF_API NerfStatus nerf_b200_occupancy_update(float* density, uint32_t* bitfield, const float* sigma, uint32_t cell_count,
                                               uint32_t update_count, uint32_t frame, uint32_t mode, float decay,
                                               float threshold, void* stream) {
    if (!density || !bitfield || cell_count == 0u || update_count > cell_count || mode > 2u) return NERF_STATUS_INVALID_USAGE;
    if (mode == 2u && update_count && !sigma) return NERF_STATUS_INVALID_USAGE;
    nb::OccupancyArgs a{};
    a.density = density;
    a.bitfield = bitfield;
    a.occ_sigma = sigma;
    a.cell_count = cell_count;
    a.update_count = update_count;
    a.decay = decay;
    a.threshold = threshold;
    a.direct = 1;
    a.mode = mode;
    a.frame = frame;
    return nb::cuda_status(nb::launch_occupancy_update(a, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
