// hs_op_linear_act_noalloc: the linear op of hs_op_linear_act (int8 x int8 -> int32, per-channel
// requant to int8, or the raw int32 accumulators) for callers that must not allocate device
// memory at call time. It has no counterpart in the reference.
//
// Who cannot allocate: a process whose device memory is already handed out by another allocator
// (a serving engine that reserves most of HBM at start-up, or torch's caching allocator holding
// freed blocks) gets an out-of-memory error from a call-time cudaMalloc even though the op needs
// only a few MiB; and a caller whose other streams run latency-bound work cannot take the
// device-wide synchronisation that cudaFree implies. This entry point instead stages the padded
// operands, the per-channel parameters, the kernel's error word and the result in one file-scope
// __device__ array of HS_STATIC_SCRATCH_BYTES (32 MiB), which every GPU that loads the library
// holds until the process exits. It calls no cudaMalloc, cudaFree or other allocating routine.
//
// Set-up: the first call on a device (with that device current) resolves the array's address
// with cudaGetSymbolAddress, which loads the module on that device, and creates the library's
// own non-blocking stream for that device; make that first call before any stream capture
// begins. Every call then runs on that stream (asynchronous memset and copies, the launch, one
// stream synchronisation), never on the legacy default stream, so it does not wait on the
// caller's other blocking streams and they do not wait on it. Every call shares the one array
// and it keeps the last call's contents, so each call first clears the padding that the GEMM
// reads as zeros. Calls that overlap on the GPU (from several host threads on one device) race on
// the array; serialise them. Shapes whose staging needs more than the array holds are refused
// with HS_UNSUPPORTED.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "../../include/hardshell_b200.h"
#include "hs_device.hpp"
#include "hs_kernels.cuh"

using namespace hs;

// Defined in hs_runtime.cu.
extern "C" int hs_internal_tmap(hs_dev* dev, void* tm, const void* base, uint64_t rows, uint64_t cols,
                                uint32_t box_rows);
extern "C" int hs_internal_dev_info(hs_dev* dev, int* num_sms, int** d_err);
extern "C" int hs_internal_fail(int code, const char* msg);

static __device__ __align__(256) uint8_t g_static_scratch[HS_STATIC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
uint8_t* g_scratch_ptr[kMaxDevices] = {};
cudaStream_t g_stream[kMaxDevices] = {};

uint64_t align256(uint64_t x) { return (x + 255) & ~uint64_t(255); }

// The array's device address on the current device and the library's stream there, both made
// once per device.
int scratch_of_current_device(uint8_t** out, cudaStream_t* stream) {
    int ord = 0;
    cudaError_t e = cudaGetDevice(&ord);
    if (e != cudaSuccess) return hs_internal_fail(HS_CUDA, cudaGetErrorString(e));
    if (ord < 0 || ord >= kMaxDevices) return hs_internal_fail(HS_UNSUPPORTED, "device ordinal out of range");
    std::lock_guard<std::mutex> lock(g_setup_mu);
    if (!g_scratch_ptr[ord]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_static_scratch);
        if (e != cudaSuccess)
            return hs_internal_fail(HS_CUDA, (std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e)).c_str());
        cudaStream_t st = nullptr;
        e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
        if (e != cudaSuccess)
            return hs_internal_fail(HS_CUDA, (std::string("cudaStreamCreateWithFlags: ") + cudaGetErrorString(e)).c_str());
        g_stream[ord] = st;
        g_scratch_ptr[ord] = static_cast<uint8_t*>(p);
    }
    *out = g_scratch_ptr[ord];
    *stream = g_stream[ord];
    return HS_OK;
}

}  // namespace

#define NA_CK(call)                                                                                 \
    do {                                                                                            \
        cudaError_t e_ = (call);                                                                    \
        if (e_ != cudaSuccess)                                                                      \
            return hs_internal_fail(HS_CUDA, (std::string(#call) + ": " + cudaGetErrorString(e_)).c_str()); \
    } while (0)

extern "C" int hs_op_linear_act_noalloc(hs_dev* dev, int path, const int8_t* A, const int8_t* W,
                                        const int32_t* bias, const int32_t* mult, uint32_t shift, uint32_t M,
                                        uint32_t N, uint32_t K, int8_t* out8, int32_t* raw32) {
    if (!dev || !A || !W || (!raw32 && (!bias || !mult || !out8))) return hs_internal_fail(HS_BAD_ARGUMENT, "null argument");
    if (M == 0 || N == 0 || K == 0 || K > 65536) return hs_internal_fail(HS_UNSUPPORTED, "shape out of range");
    if (path == 0 && N % 16 != 0)
        return hs_internal_fail(HS_UNSUPPORTED, "the tensor-core path needs N % 16 == 0 for aligned stores");
    auto up = [](uint64_t x, uint64_t m) { return (x + m - 1) / m * m; };
    const uint64_t Mp = up(M, TILE_M), Np = up(N, TILE_N), Kp = up(K, TILE_K);
    // Layout: error word | A [Mp, Kp] | W [Np, Kp] | bias [Np] | mult [Np] | result [M, N].
    const uint64_t off_a = 256;
    const uint64_t off_w = off_a + align256(Mp * Kp);
    const uint64_t off_b = off_w + align256(Np * Kp);
    const uint64_t off_m = off_b + align256(4 * Np);
    const uint64_t off_o = off_m + align256(4 * Np);
    const uint64_t need = off_o + align256((uint64_t)M * N * (raw32 ? 4 : 1));
    if (need > HS_STATIC_SCRATCH_BYTES)
        return hs_internal_fail(HS_UNSUPPORTED, ("the op needs " + std::to_string(need) +
                                                 " bytes of staging; the static scratch holds " +
                                                 std::to_string((uint64_t)HS_STATIC_SCRATCH_BYTES))
                                                    .c_str());
    int num_sms = 0;
    int* unused_err = nullptr;
    int rc = hs_internal_dev_info(dev, &num_sms, &unused_err);  // makes the device current
    if (rc) return rc;
    uint8_t* base = nullptr;
    cudaStream_t st = nullptr;
    if ((rc = scratch_of_current_device(&base, &st))) return rc;
    int* d_err = reinterpret_cast<int*>(base);
    int8_t* da = reinterpret_cast<int8_t*>(base + off_a);
    int8_t* dw = reinterpret_cast<int8_t*>(base + off_w);
    int32_t* db = reinterpret_cast<int32_t*>(base + off_b);
    int32_t* dm = reinterpret_cast<int32_t*>(base + off_m);

    // The GEMM reads the padding of A, W, bias and mult, which hold the previous call's data.
    NA_CK(cudaMemsetAsync(base, 0, off_o, st));
    NA_CK(cudaMemcpy2DAsync(da, Kp, A, K, K, M, cudaMemcpyHostToDevice, st));
    NA_CK(cudaMemcpy2DAsync(dw, Kp, W, K, K, N, cudaMemcpyHostToDevice, st));
    if (!raw32) {
        NA_CK(cudaMemcpyAsync(db, bias, 4 * (size_t)N, cudaMemcpyHostToDevice, st));
        NA_CK(cudaMemcpyAsync(dm, mult, 4 * (size_t)N, cudaMemcpyHostToDevice, st));
    }
    LinearDev L{dw, (int)N, (int)K, (int)Np, (int)Kp, db, dm, (int)shift};
    EpiArgs e{};
    e.R = (int)M;
    e.N = (int)N;
    e.b = db;
    e.m = dm;
    e.s = (int)shift;
    e.ldo = (int)N;
    if (raw32) e.out32 = reinterpret_cast<int32_t*>(base + off_o);
    else e.out8 = reinterpret_cast<int8_t*>(base + off_o);
    const int mode = raw32 ? EPI_RAW : EPI_ACT;
    if (path == 0) {
        alignas(128) CUtensorMap ta, tb;
        if ((rc = hs_internal_tmap(dev, &ta, da, Mp, Kp, TILE_M)) || (rc = hs_internal_tmap(dev, &tb, dw, Np, Kp, TILE_N)))
            return rc;
        launch_gemm_tc(mode, &ta, &tb, nullptr, (int)M, (int)Np, (int)Kp, e, num_sms, d_err, st);
    } else {
        launch_gemm_simple(mode, da, (int)Kp, (int)M, L, e, st);
    }
    NA_CK(cudaGetLastError());
    NA_CK(cudaStreamSynchronize(st));
    int herr = 0;
    NA_CK(cudaMemcpyAsync(&herr, d_err, sizeof(int), cudaMemcpyDeviceToHost, st));
    NA_CK(cudaStreamSynchronize(st));
    if (herr) return hs_internal_fail(HS_CUDA, ("a kernel wait timed out (code " + std::to_string(herr) + ")").c_str());
    if (raw32) NA_CK(cudaMemcpyAsync(raw32, base + off_o, 4 * (size_t)M * N, cudaMemcpyDeviceToHost, st));
    else NA_CK(cudaMemcpyAsync(out8, base + off_o, (size_t)M * N, cudaMemcpyDeviceToHost, st));
    NA_CK(cudaStreamSynchronize(st));
    return HS_OK;
}
