// peer.cu -- one-shot all-reduce over peer memory (NVLink / NVSwitch) for the
// row-parallel down projection of the tensor-parallel MLP.
//
// Each rank's down projection writes its partial [M, H] sum into a buffer
// that every rank can address (the allocation mapped into the other ranks'
// processes through legacy CUDA IPC handles: plain peer memory over NVLink,
// no NVLink-SHARP object).  spark_peer_allreduce then gives every
// rank the full sum without NCCL:
//   1. CTA b of rank r publishes "partial ready" to CTA b of every rank
//      (a release store of a per-CTA epoch into each rank's flag array at
//      [b][r], system scope) and waits, bounded, until every rank's CTA b
//      has published the same epoch into its own flags;
//   2. CTA b sums its slice of the elements over ranks 0..W-1 in that order
//      (fp32; identical bits on every rank) and writes the local output.
// A rank's partial is complete when any of its CTAs publishes: the partial
// was written by an earlier kernel on the same stream, made visible system-
// wide before the flag store.  Buffers alternate between two calls: when a
// rank may overwrite buffer k again (two calls later), the barrier of the
// call in between has shown that every rank finished the kernel that read
// it.  Epochs are per-CTA device counters, so the kernel replays inside CUDA
// graphs; every rank must issue the same sequence of calls.
#include <cuda.h>
#include <string.h>

#include <algorithm>

#include "common.cuh"

namespace spark {
namespace {

// Enough threads that every one handles about one 8-element group of a
// config-4 partial (64 x 4096): the peer loads are all in flight at once
// instead of paying the NVLink latency once per loop iteration.
constexpr int kPeerCtas = 128;         // same on every rank: the flag arrays are [kPeerCtas][world]
constexpr int kPeerThreads = 256;
constexpr uint64_t kPeerWaitNs = 2000000000ull;

struct PeerPtrs {
    const void* buf[SPARK_MAX_PEERS];
    int* flags[SPARK_MAX_PEERS];
};

__device__ __forceinline__ void st_release_sys(int* p, int v) {
    asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
    int v;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ float load_elem(const void* p, int dtype, int64_t i) {
    return dtype == SPARK_DTYPE_F32 ? reinterpret_cast<const float*>(p)[i]
                                    : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}

__global__ void __launch_bounds__(kPeerThreads) k_peer_allreduce(const PeerPtrs pp, int world, int rank, int64_t n,
                                                                 int in_dtype, void* __restrict__ out, int out_dtype,
                                                                 int* __restrict__ epochs, int* __restrict__ err) {
    __shared__ int ok_s;
    const int b = blockIdx.x;
    if (threadIdx.x == 0) {
        const int e = epochs[b] + 1;
        epochs[b] = e;
        // every write of this rank's partial (earlier kernels on this stream)
        // is visible system-wide before the flag
        __threadfence_system();
        for (int r = 0; r < world; ++r) st_release_sys(pp.flags[r] + b * world + rank, e);
        int ok = 1;
        const int* mine = pp.flags[rank] + b * world;
        uint64_t deadline = 0;
        for (int r = 0; r < world && ok; ++r) {
            while (ld_acquire_sys(mine + r) - e < 0) {
                if (deadline == 0) deadline = globaltimer_ns() + kPeerWaitNs;
                if (globaltimer_ns() > deadline) {
                    ok = 0;
                    break;
                }
            }
        }
        if (!ok) report_device_error(err, 5);
        ok_s = ok;
    }
    __syncthreads();
    if (!ok_s) return;
    // this CTA's slice, in 8-element groups
    const int64_t groups = (n + 7) / 8;
    const int64_t g0 = groups * b / gridDim.x, g1 = groups * (b + 1) / gridDim.x;
    for (int64_t g = g0 + threadIdx.x; g < g1; g += blockDim.x) {
        float acc[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[k] = 0.0f;
        const int64_t i0 = g * 8;
        if (i0 + 8 <= n && in_dtype == SPARK_DTYPE_BF16) {
            for (int r = 0; r < world; ++r) {
                const uint4 v = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(pp.buf[r]) + i0);
                const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    acc[2 * k] += __uint_as_float(w[k] << 16);
                    acc[2 * k + 1] += __uint_as_float(w[k] & 0xffff0000u);
                }
            }
        } else {
            for (int r = 0; r < world; ++r)
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    if (i0 + k < n) acc[k] += load_elem(pp.buf[r], in_dtype, i0 + k);
        }
#pragma unroll
        for (int k = 0; k < 8; ++k)
            if (i0 + k < n) store_from_float(out, out_dtype, i0 + k, acc[k]);
    }
}

}  // namespace
}  // namespace spark

using namespace spark;

extern "C" {

int spark_peer_flags_count(int world) { return kPeerCtas * world; }

// Sharing a device buffer with the other ranks of one node (legacy CUDA IPC:
// a plain peer mapping, no NVLink-SHARP object).  The handle names the whole
// allocation that holds `ptr` (a caching allocator hands out pieces of larger
// blocks), so the offset of `ptr` inside it travels along.
int spark_ipc_handle(const void* ptr, void* handle, int64_t* offset) {
    SPARK_REQUIRE(ptr && handle && offset, SPARK_ERR_INVALID, "spark_ipc_handle: null pointer");
    static_assert(sizeof(cudaIpcMemHandle_t) == SPARK_IPC_HANDLE_BYTES, "IPC handle size");
    using GetRange = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
    static GetRange get_range = nullptr;
    if (!get_range) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        cudaError_t e = cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &fn, 12000, cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
            return set_error(SPARK_ERR_DEVICE, "cuMemGetAddressRange unavailable");
        get_range = reinterpret_cast<GetRange>(fn);
    }
    CUdeviceptr base = 0;
    size_t size = 0;
    if (get_range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
        return set_error(SPARK_ERR_INVALID, "spark_ipc_handle: not a device allocation");
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
    if (e != cudaSuccess) return set_error((int)e, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
    memcpy(handle, &h, sizeof(h));
    *offset = (int64_t)(reinterpret_cast<CUdeviceptr>(ptr) - base);
    return SPARK_OK;
}

int spark_ipc_open(const void* handle, int64_t offset, void** ptr) {
    SPARK_REQUIRE(handle && ptr && offset >= 0, SPARK_ERR_INVALID, "spark_ipc_open: null pointer");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void* base = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return set_error((int)e, "cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
    *ptr = static_cast<uint8_t*>(base) + offset;
    return SPARK_OK;
}

int spark_ipc_close(void* ptr, int64_t offset) {
    SPARK_REQUIRE(ptr && offset >= 0, SPARK_ERR_INVALID, "spark_ipc_close: null pointer");
    cudaError_t e = cudaIpcCloseMemHandle(static_cast<uint8_t*>(ptr) - offset);
    if (e != cudaSuccess) return set_error((int)e, "cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
    return SPARK_OK;
}

int spark_peer_allreduce(const void* const* bufs, int* const* flags, int world, int rank, int64_t n, int in_dtype,
                         void* out, int out_dtype, int* epochs, int* err, void* stream) {
    SPARK_REQUIRE(bufs && flags && out && epochs && err, SPARK_ERR_INVALID, "spark_peer_allreduce: null pointer");
    SPARK_REQUIRE(world >= 1 && world <= SPARK_MAX_PEERS && rank >= 0 && rank < world && n >= 0, SPARK_ERR_INVALID,
                  "spark_peer_allreduce: world %d rank %d n %lld", world, rank, (long long)n);
    SPARK_REQUIRE(in_dtype == SPARK_DTYPE_F32 || in_dtype == SPARK_DTYPE_BF16, SPARK_ERR_INVALID,
                  "spark_peer_allreduce: partials must be fp32 or bf16");
    SPARK_REQUIRE(out_dtype == SPARK_DTYPE_F32 || out_dtype == SPARK_DTYPE_BF16 || out_dtype == SPARK_DTYPE_F16,
                  SPARK_ERR_INVALID, "spark_peer_allreduce: bad output dtype %d", out_dtype);
    PeerPtrs pp = {};
    for (int r = 0; r < world; ++r) {
        SPARK_REQUIRE(bufs[r] && flags[r] && aligned(bufs[r], 16), SPARK_ERR_ALIGNMENT,
                      "spark_peer_allreduce: rank %d buffer null or not 16-byte aligned", r);
        pp.buf[r] = bufs[r];
        pp.flags[r] = flags[r];
    }
    k_peer_allreduce<<<kPeerCtas, kPeerThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        pp, world, rank, n, in_dtype, out, out_dtype, epochs, err);
    return check_launch("spark_peer_allreduce");
}

}  // extern "C"
