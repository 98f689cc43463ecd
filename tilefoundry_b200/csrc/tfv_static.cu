// Periodic verification without any device allocation.
//
// Some callers cannot call cudaMalloc: a search process embedded in a host framework that
// owns all device memory through its own pooled allocator, or a latency-sensitive caller
// that must not trigger cudaMalloc/cudaFree because those calls can synchronize the whole
// device and stall every other stream. tfv_verify_periodic_static serves them: it runs
// the same frame analysis, sync-program compilation and verification kernels as
// tfv_analyze_frames + tfv_verify_periodic, but its frame table (the scratch those kernels
// share) is the file-scope array below instead of caller-provided memory.
//
// The array is TFV_STATIC_TABLE_BYTES long and every GPU that loads the library holds it
// until the process exits. Its device address is looked up once per device, on the first
// call for that device, with the device current; make that first call before any stream
// capture. Each later call checks that the cached address is still device memory of that
// device (cudaPointerGetAttributes, a host-side query) and looks it up again when it is not,
// which happens only after the device's context was reset (cudaDeviceReset): the module is
// then loaded anew and the array may sit elsewhere. Every call shares the one array and
// leaves its contents behind, so calls whose work overlaps on the GPU (different streams, or
// different host threads) race; the kernels overwrite every entry they later read, so
// nothing needs clearing between calls.
#include <mutex>

#include "tfv_device.cuh"

namespace {

static __device__ __align__(256) unsigned char g_frame_table[TFV_STATIC_TABLE_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
void* g_table_address[kMaxDevices] = {};

}  // namespace

// Defined in tfv_api.cu: the shared argument checks and launch sequence.
int tfv_internal_periodic_with_table(const tfv_problem* p, const tfv_frames* frames, void* table, size_t table_bytes,
                                     const tfv_periodic_batch* b, const tfv_results* r, void* stream, bool analyze);
int tfv_internal_device(const tfv_problem* p);
int tfv_internal_fail(int code, const char* message);

extern "C" int tfv_verify_periodic_static(const tfv_problem* problem, const tfv_frames* frames,
                                          const tfv_periodic_batch* batch, const tfv_results* results, void* stream) {
    if (!problem || !frames) return tfv_internal_fail(TFV_ERR_INVALID_ARGUMENT, "problem and frames must not be NULL");
    const int device = tfv_internal_device(problem);
    if (device < 0 || device >= kMaxDevices) return tfv_internal_fail(TFV_ERR_UNSUPPORTED, "device ordinal out of range");
    void* table = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_setup_mutex);
        if (g_table_address[device]) {  // still this device's memory? (not after a context reset)
            cudaPointerAttributes attr{};
            const bool valid = cudaPointerGetAttributes(&attr, g_table_address[device]) == cudaSuccess &&
                               attr.type == cudaMemoryTypeDevice && attr.device == device;
            if (!valid) {
                cudaGetLastError();  // clear a lookup error of the stale address
                g_table_address[device] = nullptr;
            }
        }
        if (!g_table_address[device]) {
            int previous = 0;
            if (cudaGetDevice(&previous) != cudaSuccess) return tfv_internal_fail(TFV_ERR_CUDA, "cudaGetDevice failed");
            if (previous != device && cudaSetDevice(device) != cudaSuccess)
                return tfv_internal_fail(TFV_ERR_CUDA, "cannot select the problem's device");
            void* address = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&address, g_frame_table);
            if (previous != device) cudaSetDevice(previous);
            if (e != cudaSuccess || !address)
                return tfv_internal_fail(TFV_ERR_CUDA, "cudaGetSymbolAddress of the static frame table failed");
            g_table_address[device] = address;
        }
        table = g_table_address[device];
    }
    return tfv_internal_periodic_with_table(problem, frames, table, TFV_STATIC_TABLE_BYTES, batch, results, stream, true);
}
