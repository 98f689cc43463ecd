// Periodic-candidate verification fed by TMA tiles (sm_100a): kernels and launchers.
// The device code is in tfv_periodic_tma.cuh.
#include <climits>
#include <cstdint>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "tfv_periodic_tma.cuh"

namespace tfv {

namespace {

constexpr int kMaxTmaOps = 256;  // TMA box height limit

template <int kBodyRows, bool kSweep>
__global__ void __launch_bounds__(kTile) verify_periodic_tma_kernel(DevProblem p, DevFrames fr, FrameTable ft,
                                                                     DevPeriodic b, DevResults out, int n_tiles,
                                                                     const __grid_constant__ CUtensorMap map_p,
                                                                     const __grid_constant__ CUtensorMap map_o) {
    tma_verify_body<kBodyRows, kSweep, NoSpec>(p, fr, ft, b, out, n_tiles, &map_p, &map_o, -1, DeltaTable{});
}

}  // namespace

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
    return fn;
}

bool make_map(CUtensorMap* map, const int16_t* base, long long n, long long stride, int N) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(n), static_cast<cuuint64_t>(N)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(stride) * sizeof(int16_t)};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(kTile), static_cast<cuuint32_t>(N)};
    cuuint32_t elem[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<int16_t*>(base), dims, strides, box, elem,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Tiles, per-op constants, the mbarrier (16 bytes) and the warps' capacity-check records.
size_t tma_smem_bytes(const DevProblem& p) { return tma_body_smem_bytes(p, 1, 1, false); }

bool periodic_tma_supported(const DevProblem& p, const DevPeriodic& b) {
    const auto aligned = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
    return p.n_ops <= kMaxTmaOps && p.iterations <= kMaxProgDistance && b.stride % 8 == 0 && aligned(b.prologue_delta) &&
           aligned(b.offset_delta) && b.n < (1LL << 31) && encode_fn() != nullptr;
}

namespace {

template <int kBodyRows, bool kSweep>
cudaError_t launch_tma(const DevProblem& p, const DevFrames& f, FrameTable t, const DevPeriodic& b, DevResults r,
                       int sm_count, cudaStream_t stream, const CUtensorMap& map_p, const CUtensorMap& map_o) {
    auto kernel = verify_periodic_tma_kernel<kBodyRows, kSweep>;
    const size_t smem = tma_smem_bytes(p);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kTile, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    const long long tiles = (b.n + kTile - 1) / kTile;
    const long long cap = static_cast<long long>(sm_count) * per_sm;
    const int grid = static_cast<int>(tiles < cap ? tiles : cap);
    kernel<<<grid, kTile, smem, stream>>>(p, f, t, b, r, static_cast<int>(tiles), map_p, map_o);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_verify_periodic_tma(const DevProblem& p, const DevFrames& f, FrameTable t, const DevPeriodic& b,
                                       DevResults r, int sm_count, cudaStream_t stream) {
    if (b.n <= 0) return cudaSuccess;
    CUtensorMap map_p, map_o;
    if (!make_map(&map_p, b.prologue_delta, b.n, b.stride, p.n_ops) ||
        !make_map(&map_o, b.offset_delta, b.n, b.stride, p.n_ops))
        return cudaErrorInvalidValue;
    if (b.n_ii > 1) {
        if (p.iterations >= 3) return launch_tma<2, true>(p, f, t, b, r, sm_count, stream, map_p, map_o);
        if (p.iterations == 2) return launch_tma<1, true>(p, f, t, b, r, sm_count, stream, map_p, map_o);
        return launch_tma<0, true>(p, f, t, b, r, sm_count, stream, map_p, map_o);
    }
    if (p.iterations >= 3) return launch_tma<2, false>(p, f, t, b, r, sm_count, stream, map_p, map_o);
    if (p.iterations == 2) return launch_tma<1, false>(p, f, t, b, r, sm_count, stream, map_p, map_o);
    return launch_tma<0, false>(p, f, t, b, r, sm_count, stream, map_p, map_o);
}

}  // namespace tfv
