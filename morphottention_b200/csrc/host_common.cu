// host_common.cu -- implementation of the host helpers (errors, launch counts,
// tensor maps, device facts) and the definition of the device status word.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "host_common.h"

namespace morpho {

// Device status word written by kernels whose bounded waits expire (one per device,
// since a __device__ variable has an instance in every device context).
__device__ uint32_t g_device_status = 0u;

namespace {
thread_local char t_err[1024] = {0};
thread_local int t_launches = 0;

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, []() {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

constexpr int kMaxDevices = 64;
DeviceInfo g_info[kMaxDevices];
std::mutex g_info_mu;
}  // namespace

namespace {
struct ProfRec {
    const char* name;
    cudaEvent_t start, stop;
};
// The switch and the selection are process-wide and may be changed from any host thread
// while others launch: the switch is atomic, the selected name is guarded by a mutex (taken
// only while timing is on).  The records themselves are per host thread.
std::atomic<bool> g_prof_on{false};
std::mutex g_prof_mu;
std::string g_prof_only;  // empty: every launch is timed
thread_local std::vector<ProfRec> t_prof;
thread_local std::vector<cudaEvent_t> t_event_pool;
thread_local cudaEvent_t t_pending = nullptr;

cudaEvent_t take_event() {
    if (!t_event_pool.empty()) {
        cudaEvent_t e = t_event_pool.back();
        t_event_pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
    return e;
}
}  // namespace

void prof_enable(bool on) { g_prof_on.store(on); }

void prof_select(const char* name) {
    std::lock_guard<std::mutex> lock(g_prof_mu);
    g_prof_only = name ? name : "";
}

void prof_begin(cudaStream_t stream, const char* name) {
    if (!g_prof_on.load(std::memory_order_relaxed)) return;
    bool selected = true;
    {
        std::lock_guard<std::mutex> lock(g_prof_mu);
        selected = g_prof_only.empty() || (name != nullptr && g_prof_only == name);
    }
    if (!selected) {
        t_pending = nullptr;  // not selected: no events, prof_end records nothing
        return;
    }
    t_pending = take_event();
    if (t_pending) cudaEventRecord(t_pending, stream);
}

void prof_end(const char* name, cudaStream_t stream) {
    if (!g_prof_on.load(std::memory_order_relaxed) || t_pending == nullptr) return;
    cudaEvent_t stop = take_event();
    if (stop == nullptr) return;
    cudaEventRecord(stop, stream);
    t_prof.push_back({name, t_pending, stop});
    t_pending = nullptr;
}

int prof_collect(char* names, int name_len, float* total_ms, int* counts, int max_kernels) {
    std::map<std::string, std::pair<double, int>> agg;
    std::vector<std::string> order;
    for (auto& r : t_prof) {
        float ms = 0.f;
        cudaEventSynchronize(r.stop);
        cudaEventElapsedTime(&ms, r.start, r.stop);
        auto it = agg.find(r.name);
        if (it == agg.end()) {
            order.push_back(r.name);
            agg[r.name] = {ms, 1};
        } else {
            it->second.first += ms;
            it->second.second += 1;
        }
        t_event_pool.push_back(r.start);
        t_event_pool.push_back(r.stop);
    }
    t_prof.clear();
    int n = 0;
    for (auto& k : order) {
        if (n >= max_kernels) break;
        snprintf(names + static_cast<size_t>(n) * name_len, name_len, "%s", k.c_str());
        total_ms[n] = static_cast<float>(agg[k].first);
        counts[n] = agg[k].second;
        ++n;
    }
    return n;
}

int set_error(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_err, sizeof(t_err), fmt, ap);
    va_end(ap);
    return code;
}

const char* last_error() { return t_err; }
void clear_error() { t_err[0] = 0; }

void reset_launch_count() { t_launches = 0; }
void count_launch(int n) { t_launches += n; }
int launch_count() { return t_launches; }

int make_tmap(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int rank, const uint64_t* dims,
              const uint64_t* row_strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle) {
    EncodeTiledFn fn = encode_fn();
    if (fn == nullptr) return set_error(MORPHO_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
    cuuint64_t gdim[5];
    cuuint64_t gstride[4];
    cuuint32_t bdim[5];
    cuuint32_t estride[5];
    for (int i = 0; i < rank; ++i) {
        gdim[i] = dims[i];
        bdim[i] = box[i];
        estride[i] = 1;
    }
    for (int i = 0; i + 1 < rank; ++i) gstride[i] = row_strides_bytes[i];
    CUresult r = fn(map, dtype, static_cast<cuuint32_t>(rank), const_cast<void*>(base), gdim, gstride, bdim, estride,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return set_error(MORPHO_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d): rank %d dims %llu x %llu box %u x %u",
                         static_cast<int>(r), rank, static_cast<unsigned long long>(dims[0]),
                         static_cast<unsigned long long>(rank > 1 ? dims[1] : 1), box[0], rank > 1 ? box[1] : 1);
    return MORPHO_OK;
}

static CUtensorMapSwizzle swizzle_for_bytes(uint32_t inner_bytes) {
    if (inner_bytes >= 128) return CU_TENSOR_MAP_SWIZZLE_128B;
    if (inner_bytes >= 64) return CU_TENSOR_MAP_SWIZZLE_64B;
    return CU_TENSOR_MAP_SWIZZLE_32B;
}

int make_tmap_2d_f16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows,
                     uint32_t box_cols) {
    const uint64_t dims[2] = {cols, rows};
    const uint64_t strides[1] = {ld * 2};
    const uint32_t box[2] = {box_cols, box_rows};
    return make_tmap(map, base, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, dims, strides, box,
                     swizzle_for_bytes(box_cols * 2));
}

int make_tmap_3d_f16(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t stride1,
                     uint64_t stride2, uint32_t box0, uint32_t box1) {
    const uint64_t dims[3] = {d0, d1, d2};
    const uint64_t strides[2] = {stride1 * 2, stride2 * 2};
    const uint32_t box[3] = {box0, box1, 1};
    return make_tmap(map, base, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, dims, strides, box, swizzle_for_bytes(box0 * 2));
}

int make_tmap_2d_f32(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows,
                     uint32_t box_cols) {
    const uint64_t dims[2] = {cols, rows};
    const uint64_t strides[1] = {ld * 4};
    const uint32_t box[2] = {box_cols, box_rows};
    return make_tmap(map, base, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_NONE);
}

int current_device_info(DeviceInfo* out) {
    int dev = 0;
    MORPHO_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return set_error(MORPHO_ERR_DEVICE, "device ordinal %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_info_mu);
    DeviceInfo& info = g_info[dev];
    if (info.device != dev) {
        DeviceInfo d;
        d.device = dev;
        MORPHO_CUDA_TRY(cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev));
        MORPHO_CUDA_TRY(cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev));
        MORPHO_CUDA_TRY(cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev));
        MORPHO_CUDA_TRY(cudaDeviceGetAttribute(&d.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
        void* addr = nullptr;
        MORPHO_CUDA_TRY(cudaGetSymbolAddress(&addr, g_device_status));
        d.status = static_cast<uint32_t*>(addr);
        info = d;
    }
    if (info.cc_major != 10 || info.cc_minor != 0)
        return set_error(MORPHO_ERR_DEVICE, "device %d is sm_%d%d; these kernels are built for sm_100a only", dev,
                         info.cc_major, info.cc_minor);
    *out = info;
    return MORPHO_OK;
}

}  // namespace morpho
