// host_common.h -- host helpers shared by the sm_100a launchers: thread-local error
// messages, CUDA error checks, launch counting and TMA tensor-map encoding.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/morpho_sm100.h"

namespace morpho {

// Record a printf-style message as the calling thread's last error; returns `code`.
int set_error(int code, const char* fmt, ...);
const char* last_error();
void clear_error();

// Kernel launches made by the current entry point on this thread.
void reset_launch_count();
void count_launch(int n = 1);
int launch_count();

// Optional per-launch CUDA-event timing (off by default): prof_begin records a start
// event on the launching stream, prof_end a stop event tagged with the kernel name.
void prof_begin(cudaStream_t stream, const char* name);
void prof_end(const char* name, cudaStream_t stream);
void prof_enable(bool on);
// Time only the launches of this kernel name (NULL or "": every launch).
void prof_select(const char* name);
// Aggregate the recorded launches per kernel name (synchronises the events) and clear.
int prof_collect(char* names, int name_len, float* total_ms, int* counts, int max_kernels);

#define MORPHO_CUDA_TRY(expr)                                                                                 \
    do {                                                                                                      \
        cudaError_t e_ = (expr);                                                                              \
        if (e_ != cudaSuccess)                                                                                \
            return ::morpho::set_error(MORPHO_ERR_CUDA, "%s failed: %s (%s:%d)", #expr, cudaGetErrorString(e_), \
                                       __FILE__, __LINE__);                                                   \
    } while (0)

#define MORPHO_TRY(expr)           \
    do {                           \
        int rc_ = (expr);          \
        if (rc_ != MORPHO_OK)      \
            return rc_;            \
    } while (0)

// Check the last launch (and close its profiling interval; `stream` must be in scope).
#define MORPHO_LAUNCH_CHECK(name)                                                                              \
    do {                                                                                                       \
        cudaError_t e_ = cudaGetLastError();                                                                   \
        if (e_ != cudaSuccess)                                                                                 \
            return ::morpho::set_error(MORPHO_ERR_CUDA, "launch of %s failed: %s", name, cudaGetErrorString(e_)); \
        ::morpho::count_launch();                                                                              \
        ::morpho::prof_end(name, stream);                                                                      \
    } while (0)

// Tiled tensor map over a row-major fp16/fp32 tensor.  dims/box are innermost first;
// row_strides_bytes has rank-1 entries (stride of dims[1], dims[2], ...).
int make_tmap(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int rank, const uint64_t* dims,
              const uint64_t* row_strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle);

// 2D fp16 map over a [rows, cols] row-major matrix with leading dimension ld (elements),
// box {box_cols, box_rows}, swizzle chosen from box_cols*2 bytes (32/64/128).
int make_tmap_2d_f16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                     uint32_t box_rows, uint32_t box_cols);

// 3D fp16 map over [d2, d1, d0] (d0 innermost, contiguous), box {box0, box1, 1}.
int make_tmap_3d_f16(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t stride1,
                     uint64_t stride2, uint32_t box0, uint32_t box1);

// 2D fp32 map over [rows, cols] (no swizzle), box {box_cols, box_rows}.
int make_tmap_2d_f32(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                     uint32_t box_rows, uint32_t box_cols);

// Device facts of the current device (cached per device).
struct DeviceInfo {
    int device = -1;
    int sms = 0;
    int cc_major = 0;
    int cc_minor = 0;
    int smem_optin = 0;
    uint32_t* status = nullptr;  // device address of the status word
};
int current_device_info(DeviceInfo* out);

}  // namespace morpho
