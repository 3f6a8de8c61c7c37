// peer.cu -- the data-parallel weight-gradient all-reduce over NVLink peer memory, fused with
// the fp16 finalize (no reference counterpart: the reference has no multi-GPU code).
//
// Each rank of a one-node group owns an exchange region in its own device memory, which the
// other ranks map with CUDA IPC: a signal block (per source rank, the last step epoch it has
// reached, written by that rank with system-scope release stores) and two fp32 buckets used on
// alternate steps.  One kernel per step runs on the caller's communication stream once this
// rank's bucket is complete, and needs no SM to itself (no shared memory, few registers): it
// shares the SMs with the dX GEMM that runs at the same time.
//   A  publish: store epoch e in slot ready[rank] of every rank's signal block, then wait until
//      every slot ready[s] of this rank's block holds e (rank s's bucket is complete);
//   B  reduce-scatter: rank r owns chunk r of the bucket.  It sums chunk r of all W buckets
//      (peer loads over NVLink) in rank order 0, 1, .., W-1 -- the same order on every rank, so
//      every rank ends with the same bits -- into its own bucket, and writes those elements'
//      fp16 gradients (times alpha).  The last CTA to finish publishes done[rank] = e;
//   C  all-gather: once done[s] = e for every s, copy the other ranks' reduced chunks into its
//      own bucket and write their fp16 gradients.
// Why two buckets suffice without a closing barrier: rank r can only rewrite a bucket two steps
// later, after its next kernel saw every peer's ready slot of the next step, which each peer
// writes only when its kernel of this step (and with it every read of rank r's bucket) is over.
// Every wait is bounded (1 s); on expiry the kernel records a status and returns.
#include <string.h>

#include "kernels.h"
#include "sm100.cuh"

namespace morpho {
namespace {

constexpr int kPeerMaxWorld = 16;
// 128 threads: one warp per SM sub-partition, whose register share still fits beside the dX GEMM's
// three warps there (registers are allocated per sub-partition); with two warps there it did not,
// and the CTAs waited for the GEMM's SMs to empty.
constexpr int kPeerThreads = 128;
constexpr int kPeerCtas = 128;
constexpr uint32_t K_PEER = 5;  // status-word kernel id (site: 1 ready, 2 done)
// Region layout: signal block (ready[16], done[16], local CTA counter), then two buckets.
constexpr size_t kSigBytes = 256;
constexpr size_t kReadyOff = 0;
constexpr size_t kDoneOff = 64;
constexpr size_t kCounterOff = 128;

struct PeerArgs {
    const float* buf[kPeerMaxWorld];  // every rank's bucket of this step (own one local)
    uint32_t* sig[kPeerMaxWorld];     // every rank's signal block
    float* own;                       // this rank's bucket
    uint32_t* own_sig;
    uint32_t* counter;
    int rank, world;
    uint32_t epoch;
    long long chunk4;   // float4 units per rank chunk
    long long n4;       // float4 units holding data (the rest is zero padding)
    long long phi4, v4, gate4;  // fp16 segment ends in float4 units: dW_phi | dW_V | d_gate_q | d_gate_k
    float alpha;
    __half* dW_phi;
    __half* dW_V;
    __half* dgq;
    __half* dgk;
    uint32_t* status;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Bounded wait of thread t < world for slot t of this rank's block to reach the epoch; the CTA
// agrees on the outcome.
__device__ bool wait_slots(const PeerArgs& a, size_t off, uint32_t site) {
    __shared__ int failed;
    if (threadIdx.x == 0) failed = 0;
    __syncthreads();
    if (threadIdx.x < a.world) {
        const uint32_t* slot = reinterpret_cast<const uint32_t*>(reinterpret_cast<const uint8_t*>(a.own_sig) + off) +
                               threadIdx.x;
        if (static_cast<int32_t>(ld_acquire_sys(slot) - a.epoch) < 0) {
            const uint64_t t0 = global_timer_ns();
            while (static_cast<int32_t>(ld_acquire_sys(slot) - a.epoch) < 0) {
                if (global_timer_ns() - t0 > WAIT_LIMIT_NS) {
                    report_timeout(a.status, K_PEER, site);
                    failed = 1;
                    break;
                }
                __nanosleep(200);
            }
        }
    }
    __syncthreads();
    return failed == 0;
}

// Publish the epoch in slot [rank] of every rank's signal block (thread t writes rank t's).
__device__ __forceinline__ void publish(const PeerArgs& a, size_t off) {
    if (threadIdx.x < a.world) {
        uint32_t* slot = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(a.sig[threadIdx.x]) + off) + a.rank;
        st_release_sys(slot, a.epoch);
    }
}

// The reduced float4 unit u: into this rank's bucket and, scaled, into its fp16 gradient.
__device__ __forceinline__ void emit(const PeerArgs& a, long long u, float4 v) {
    __stcg(reinterpret_cast<float4*>(a.own) + u, v);
    if (u >= a.n4) return;
    __half* dst;
    if (u < a.phi4)
        dst = a.dW_phi + 4 * u;
    else if (u < a.v4)
        dst = a.dW_V + 4 * (u - a.phi4);
    else if (u < a.gate4)
        dst = a.dgq + 4 * (u - a.v4);
    else if (u < 2 * a.gate4 - a.v4)
        dst = a.dgk + 4 * (u - a.gate4);
    else
        return;  // the soft-morphology temperature gradient (fp32 only) and padding
    const __half2 lo = __floats2half2_rn(a.alpha * v.x, a.alpha * v.y);
    const __half2 hi = __floats2half2_rn(a.alpha * v.z, a.alpha * v.w);
    uint2 pk;
    pk.x = *reinterpret_cast<const uint32_t*>(&lo);
    pk.y = *reinterpret_cast<const uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(dst) = pk;
}

// Sum of unit u over the W buckets in rank order: all W loads are issued before the adds (W is a
// compile-time constant where it can be: 2, 4, 8; 0 = the group's size at run time).
template <int W>
__device__ __forceinline__ float4 rank_order_sum(const PeerArgs& a, long long u) {
    if constexpr (W > 0) {
        float4 x[W];
#pragma unroll
        for (int r = 0; r < W; ++r) x[r] = __ldcg(reinterpret_cast<const float4*>(a.buf[r]) + u);
        float4 s = x[0];
#pragma unroll
        for (int r = 1; r < W; ++r) s = make_float4(s.x + x[r].x, s.y + x[r].y, s.z + x[r].z, s.w + x[r].w);
        return s;
    } else {  // a load per step: few registers, so the kernel still fits beside the dX GEMM
        float4 s = __ldcg(reinterpret_cast<const float4*>(a.buf[0]) + u);
        for (int r = 1; r < a.world; ++r) {
            const float4 x = __ldcg(reinterpret_cast<const float4*>(a.buf[r]) + u);
            s = make_float4(s.x + x.x, s.y + x.y, s.z + x.z, s.w + x.w);
        }
        return s;
    }
}

template <int W>
__global__ void __launch_bounds__(kPeerThreads) peer_allreduce_kernel(const PeerArgs a) {
    // A: this rank's bucket is complete (stream order); publish, then wait for every rank's
    if (blockIdx.x == 0) publish(a, kReadyOff);
    if (!wait_slots(a, kReadyOff, 1)) return;

    // B: reduce chunk `rank` in rank order, two float4 units per thread per pass
    const long long c0 = static_cast<long long>(a.rank) * a.chunk4;
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < a.chunk4; i += 2 * stride) {
        const bool has1 = i + stride < a.chunk4;
        const float4 s0 = rank_order_sum<W>(a, c0 + i);
        if (has1) {
            const float4 s1 = rank_order_sum<W>(a, c0 + i + stride);
            emit(a, c0 + i, s0);
            emit(a, c0 + i + stride, s1);
        } else {
            emit(a, c0 + i, s0);
        }
    }
    // the last CTA to finish its part publishes "chunk done" (every CTA's stores are ordered
    // before its counter increment by a system-scope fence)
    __shared__ int last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        last = atomicAdd(a.counter, 1u) == gridDim.x - 1;
        if (last) {
            *a.counter = 0u;  // for the next step's launch (stream-ordered after this one)
            __threadfence_system();
        }
    }
    __syncthreads();
    if (last) publish(a, kDoneOff);

    // C: gather the other ranks' reduced chunks: one flat index space over the W - 1 chunks,
    // four units per thread per pass with their loads in flight together
    if (!wait_slots(a, kDoneOff, 2)) return;
    const long long total = static_cast<long long>(a.world - 1) * a.chunk4;
    for (long long j0 = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; j0 < total; j0 += 4 * stride) {
        long long unit[4];
        float4 v[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const long long j = j0 + q * stride;
            unit[q] = -1;
            if (j < total) {
                const long long k = j / a.chunk4;
                const int r = static_cast<int>((a.rank + 1 + k) % a.world);  // peers in a rotated order
                unit[q] = static_cast<long long>(r) * a.chunk4 + (j - k * a.chunk4);
                v[q] = __ldcg(reinterpret_cast<const float4*>(a.buf[r]) + unit[q]);
            }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q)
            if (unit[q] >= 0) emit(a, unit[q], v[q]);
    }
}

}  // namespace
}  // namespace morpho

using namespace morpho;

struct morpho_peer_group {
    int rank = 0, world = 0, device = -1;
    long long elems = 0;    // bucket elements the caller uses
    long long chunk4 = 0;   // float4 units per rank chunk
    size_t bucket_bytes = 0;
    uint8_t* region = nullptr;              // own exchange region (cudaMalloc)
    uint8_t* peer[kPeerMaxWorld] = {};      // every rank's region as mapped here (own = region)
    uint32_t epoch = 0;                     // completed all-reduces
};

namespace {

uint8_t* bucket_of(const morpho_peer_group* g, int r, uint32_t epoch) {
    return g->peer[r] + kSigBytes + (epoch & 1u) * g->bucket_bytes;
}

}  // namespace

extern "C" MORPHO_API int morpho_sm100_peer_create(int32_t rank, int32_t world, int64_t bucket_elems, void* handle_out,
                                                   char* pci_bus_id_out, morpho_peer_group_t** group) {
    clear_error();
    reset_launch_count();
    if (group == nullptr || handle_out == nullptr || pci_bus_id_out == nullptr)
        return set_error(MORPHO_ERR_INVALID, "peer_create: NULL argument");
    *group = nullptr;
    if (world < 1 || world > kPeerMaxWorld || rank < 0 || rank >= world)
        return set_error(MORPHO_ERR_INVALID, "peer_create: rank %d / world %d (1 .. %d ranks)", rank, world,
                         kPeerMaxWorld);
    if (bucket_elems <= 0) return set_error(MORPHO_ERR_INVALID, "peer_create: bucket_elems %lld", (long long)bucket_elems);
    auto* g = new morpho_peer_group();
    g->rank = rank;
    g->world = world;
    g->elems = bucket_elems;
    g->chunk4 = ((bucket_elems + 3) / 4 + world - 1) / world;
    g->bucket_bytes = static_cast<size_t>(g->chunk4) * world * 16;
    const size_t bytes = kSigBytes + 2 * g->bucket_bytes;
    cudaError_t e = cudaGetDevice(&g->device);
    if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&g->region), bytes);
    if (e == cudaSuccess) e = cudaMemset(g->region, 0, bytes);  // epochs 0, zero padding
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, g->region);
    if (e == cudaSuccess) e = cudaDeviceGetPCIBusId(pci_bus_id_out, MORPHO_PEER_PCI_ID_BYTES, g->device);
    if (e != cudaSuccess) {
        if (g->region != nullptr) cudaFree(g->region);
        delete g;
        return set_error(MORPHO_ERR_CUDA, "peer_create: %s", cudaGetErrorString(e));
    }
    static_assert(sizeof(cudaIpcMemHandle_t) == MORPHO_PEER_HANDLE_BYTES, "IPC handle size");
    memcpy(handle_out, &h, sizeof(h));
    g->peer[rank] = g->region;
    *group = g;
    return MORPHO_OK;
}

extern "C" MORPHO_API int morpho_sm100_peer_connect(morpho_peer_group_t* g, const void* handles,
                                                    const char* pci_bus_ids) {
    clear_error();
    if (g == nullptr || handles == nullptr || pci_bus_ids == nullptr)
        return set_error(MORPHO_ERR_INVALID, "peer_connect: NULL argument");
    for (int r = 0; r < g->world; ++r) {
        if (r == g->rank) continue;
        const char* id = pci_bus_ids + static_cast<size_t>(r) * MORPHO_PEER_PCI_ID_BYTES;
        int dev = -1, can = 0;
        cudaError_t e = cudaDeviceGetByPCIBusId(&dev, id);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return set_error(MORPHO_ERR_UNSUPPORTED, "peer_connect: rank %d's GPU (%s) is not visible here", r, id);
        }
        if (dev == g->device)
            return set_error(MORPHO_ERR_UNSUPPORTED, "peer_connect: rank %d uses this rank's GPU", r);
        e = cudaDeviceCanAccessPeer(&can, g->device, dev);
        if (e != cudaSuccess || !can)
            return set_error(MORPHO_ERR_UNSUPPORTED, "peer_connect: no peer access from GPU %d to GPU %d", g->device,
                             dev);
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const uint8_t*>(handles) + static_cast<size_t>(r) * MORPHO_PEER_HANDLE_BYTES, sizeof(h));
        void* p = nullptr;
        e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess)
            return set_error(MORPHO_ERR_CUDA, "peer_connect: mapping rank %d's region: %s", r, cudaGetErrorString(e));
        g->peer[r] = static_cast<uint8_t*>(p);
    }
    return MORPHO_OK;
}

extern "C" MORPHO_API float* morpho_sm100_peer_bucket(const morpho_peer_group_t* g) {
    return g == nullptr ? nullptr : reinterpret_cast<float*>(bucket_of(g, g->rank, g->epoch + 1));
}

extern "C" MORPHO_API int morpho_sm100_peer_allreduce_finalize(morpho_peer_group_t* g, const morpho_problem_t* p,
                                                               float alpha, void* dW_phi, void* d_gate_q,
                                                               void* d_gate_k, void* dW_V, void* stream_arg) {
    clear_error();
    reset_launch_count();
    if (g == nullptr) return set_error(MORPHO_ERR_INVALID, "peer_allreduce: NULL group");
    for (int r = 0; r < g->world; ++r)
        if (g->peer[r] == nullptr) return set_error(MORPHO_ERR_INVALID, "peer_allreduce: rank %d not connected", r);
    const long long D = p->D, Hm = static_cast<long long>(p->H) * p->cube_m;
    const long long n16 = D * Hm + D * D + 2 * Hm;  // the fp16 segments
    if (n16 % 4 != 0 || n16 > g->elems)
        return set_error(MORPHO_ERR_INVALID, "peer_allreduce: problem needs %lld bucket elements (group has %lld)", n16,
                         g->elems);
    if (dW_phi == nullptr || d_gate_q == nullptr || d_gate_k == nullptr || dW_V == nullptr)
        return set_error(MORPHO_ERR_INVALID, "peer_allreduce: NULL gradient pointer");
    DeviceInfo dev;
    MORPHO_TRY(current_device_info(&dev));
    if (dev.device != g->device)
        return set_error(MORPHO_ERR_INVALID, "peer_allreduce: current device %d, group created on %d", dev.device,
                         g->device);
    const uint32_t e = g->epoch + 1;
    PeerArgs a;
    memset(&a, 0, sizeof(a));
    for (int r = 0; r < g->world; ++r) {
        a.buf[r] = reinterpret_cast<const float*>(bucket_of(g, r, e));
        a.sig[r] = reinterpret_cast<uint32_t*>(g->peer[r]);
    }
    a.own = reinterpret_cast<float*>(bucket_of(g, g->rank, e));
    a.own_sig = reinterpret_cast<uint32_t*>(g->region);
    a.counter = reinterpret_cast<uint32_t*>(g->region + kCounterOff);
    a.rank = g->rank;
    a.world = g->world;
    a.epoch = e;
    a.chunk4 = g->chunk4;
    a.n4 = n16 / 4;
    a.phi4 = D * Hm / 4;
    a.v4 = a.phi4 + D * D / 4;
    a.gate4 = a.v4 + Hm / 4;
    a.alpha = alpha;
    a.dW_phi = static_cast<__half*>(dW_phi);
    a.dW_V = static_cast<__half*>(dW_V);
    a.dgq = static_cast<__half*>(d_gate_q);
    a.dgk = static_cast<__half*>(d_gate_k);
    a.status = dev.status;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_arg);
    prof_begin(stream, "peer_allreduce");
    switch (g->world) {
        case 2: peer_allreduce_kernel<2><<<kPeerCtas, kPeerThreads, 0, stream>>>(a); break;
        case 4: peer_allreduce_kernel<4><<<kPeerCtas, kPeerThreads, 0, stream>>>(a); break;
        case 8: peer_allreduce_kernel<8><<<kPeerCtas, kPeerThreads, 0, stream>>>(a); break;
        default: peer_allreduce_kernel<0><<<kPeerCtas, kPeerThreads, 0, stream>>>(a); break;
    }
    MORPHO_LAUNCH_CHECK("peer_allreduce");
    g->epoch = e;
    return MORPHO_OK;
}

extern "C" MORPHO_API int morpho_sm100_peer_destroy(morpho_peer_group_t* g) {
    clear_error();
    if (g == nullptr) return MORPHO_OK;
    int rc = MORPHO_OK;
    for (int r = 0; r < g->world; ++r) {
        if (r == g->rank || g->peer[r] == nullptr) continue;
        const cudaError_t e = cudaIpcCloseMemHandle(g->peer[r]);
        if (e != cudaSuccess) rc = set_error(MORPHO_ERR_CUDA, "peer_destroy: %s", cudaGetErrorString(e));
    }
    if (g->region != nullptr) {
        const cudaError_t e = cudaFree(g->region);
        if (e != cudaSuccess) rc = set_error(MORPHO_ERR_CUDA, "peer_destroy: %s", cudaGetErrorString(e));
    }
    delete g;
    return rc;
}
