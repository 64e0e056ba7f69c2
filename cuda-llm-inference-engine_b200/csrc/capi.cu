// C ABI (include/b2decode.h) and the reference-compatible C++ entry points
// (include/b2_reference_api.h) over the sm_100a kernels.
#include "common.cuh"
#include "b2_reference_api.h"
#include "engine_kernels.cuh"
#include <algorithm>
#include <cuda.h>
#include <mutex>
#include <set>
#include <utility>

namespace b2 {

// The library's device error word (B2_DEVERR_* bits), one per device.
__device__ unsigned int g_device_error = 0;

int decode_attn_launch(const b2_decode_attn_args* a, bool counters_zeroed, cudaStream_t st);
size_t decode_attn_workspace_size(int B, int H_q, int H_kv, int D, int max_ctx, int block_size);
int quantize_launch(int rows, int cols, const float* in, int32_t* out, float* scales, cudaStream_t st);
int gemm_launch(int M, int N, int K, const int32_t* A, const int32_t* BT, const float* sA, const float* sB,
                const float* bias, const float* residual, void* C, int epi, bool s32, cudaStream_t st,
                void* ws = nullptr, size_t ws_bytes = 0);
size_t gemm_workspace_size(int M, int N, int K);

constexpr int kMaxDevices = 64;

int num_sms_current_device() {
    static int cache[kMaxDevices] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
    if (cache[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (kernel, device). `slot` is
// unused (kept for call-site compatibility); the kernel's address identifies it.
bool set_smem_attr_once(const void* func, int bytes, int /*slot*/) {
    static std::set<std::pair<int, const void*>> done;
    static std::mutex mu;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    std::lock_guard<std::mutex> lk(mu);
    if (done.count({dev, func})) return true;
    if (cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) return false;
    done.insert({dev, func});
    return true;
}

unsigned int* device_error_ptr() {
    static unsigned int* cache[kMaxDevices] = {nullptr};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    if (!cache[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
        cache[dev] = static_cast<unsigned int*>(p);
    }
    return cache[dev];
}

bool& pdl_enabled() {
    static thread_local bool on = false;
    return on;
}

bool& weights_constant() {
    static thread_local bool on = false;
    return on;
}


static thread_local int t_last_status = B2_OK;

}  // namespace b2

using namespace b2;

// ------------------------------------------------------------------ C ABI
extern "C" {

size_t b2_decode_attn_workspace_size(int B, int H_q, int H_kv, int head_dim, int max_context_len, int block_size) {
    if (B <= 0 || H_q <= 0 || H_kv <= 0 || head_dim <= 0 || block_size <= 0 || max_context_len < 0) return 0;
    if (H_q % H_kv != 0) return 0;
    return decode_attn_workspace_size(B, H_q, H_kv, head_dim, max_context_len, block_size);
}

int b2_decode_attn(const b2_decode_attn_args* args, b2_stream_t stream) {
    // Launched with programmatic dependent launch: the kernel's first instruction waits for
    // the previous grid on the stream to complete (griddepcontrol.wait) and it reads nothing
    // before, so any producer of Q, the caches or the tables is safe; the launch overlaps
    // the previous kernel's tail (about 0.15 us per call, 1-2% on long batches).
    const bool saved = pdl_enabled();
    pdl_enabled() = true;
    const int r = decode_attn_launch(args, true, static_cast<cudaStream_t>(stream));
    pdl_enabled() = saved;
    return r;
}

int b2_quantize_fp32_to_int8(int rows, int cols, const float* input, int32_t* output_packed, float* scales,
                             b2_stream_t stream) {
    return quantize_launch(rows, cols, input, output_packed, scales, static_cast<cudaStream_t>(stream));
}

int b2_int8_gemm(int M, int N, int K, const int32_t* A_packed, const int32_t* BT_packed, const float* scale_A,
                 const float* scale_B, const float* bias, const float* residual, float* C, int epilogue,
                 b2_stream_t stream) {
    // programmatic dependent launch: set-up overlaps the previous kernel; no global memory is
    // read before the kernel waits for it
    PdlOn pdl;
    return gemm_launch(M, N, K, A_packed, BT_packed, scale_A, scale_B, bias, residual, C, epilogue, false,
                       static_cast<cudaStream_t>(stream));
}

size_t b2_int8_gemm_workspace_size(int M, int N, int K) {
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    return gemm_workspace_size(M, N, K);
}

int b2_int8_gemm_ws(int M, int N, int K, const int32_t* A_packed, const int32_t* BT_packed, const float* scale_A,
                    const float* scale_B, const float* bias, const float* residual, float* C, int epilogue,
                    void* workspace, size_t workspace_bytes, b2_stream_t stream) {
    if (workspace && ((uintptr_t)workspace & 255)) return B2_ERR_INVALID;
    PdlOn pdl;
    return gemm_launch(M, N, K, A_packed, BT_packed, scale_A, scale_B, bias, residual, C, epilogue, false,
                       static_cast<cudaStream_t>(stream), workspace, workspace_bytes);
}

int b2_int8_gemm_s32(int M, int N, int K, const int32_t* A_packed, const int32_t* BT_packed, int32_t* C_acc,
                     b2_stream_t stream) {
    PdlOn pdl;
    return gemm_launch(M, N, K, A_packed, BT_packed, nullptr, nullptr, nullptr, nullptr, C_acc, B2_EPI_PLAIN, true,
                       static_cast<cudaStream_t>(stream));
}

int b2_int8_gemm_s32_ws(int M, int N, int K, const int32_t* A_packed, const int32_t* BT_packed, int32_t* C_acc,
                        void* workspace, size_t workspace_bytes, b2_stream_t stream) {
    if (workspace && ((uintptr_t)workspace & 255)) return B2_ERR_INVALID;
    PdlOn pdl;
    return gemm_launch(M, N, K, A_packed, BT_packed, nullptr, nullptr, nullptr, nullptr, C_acc, B2_EPI_PLAIN, true,
                       static_cast<cudaStream_t>(stream), workspace, workspace_bytes);
}

int b2_layernorm(int rows, int cols, const float* x, const float* gamma, const float* beta, float eps, float* out,
                 int32_t* q_packed, float* scales, b2_stream_t stream) {
    if (rows < 0 || cols <= 0) return B2_ERR_INVALID;
    if (rows == 0) return B2_OK;
    if (!x || !gamma || !beta || (!out && !q_packed) || (q_packed && !scales)) return B2_ERR_INVALID;
    if ((cols & 3) || cols > 8192) return B2_ERR_UNSUPPORTED;
    return launch_ln_quant(rows, cols, x, gamma, beta, eps, q_packed, scales, out, static_cast<cudaStream_t>(stream));
}

unsigned int b2_get_device_error(int clear) {
    unsigned int v = 0;
    if (cudaDeviceSynchronize() != cudaSuccess) return 0xffffffffu;
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v)) != cudaSuccess) return 0xffffffffu;
    if (clear) {
        const unsigned int z = 0;
        cudaMemcpyToSymbol(g_device_error, &z, sizeof(z));
    }
    return v;
}

int b2_last_status(void) { return t_last_status; }

const char* b2_status_string(int status) {
    switch (status) {
        case B2_OK: return "ok";
        case B2_ERR_INVALID: return "invalid argument";
        case B2_ERR_UNSUPPORTED: return "unsupported shape";
        case B2_ERR_WORKSPACE: return "workspace missing or too small";
        case B2_ERR_CUDA: return "CUDA runtime error";
        case B2_ERR_TIMEOUT: return "peer timeout";
        default: return "unknown status";
    }
}

int b2_version(void) { return 100; }

}  // extern "C"

// ------------------------------------------------------------------ reference-compatible C++ API
// Same names and parameter lists as the reference; launches go to the legacy default
// stream as the reference's do. Errors, which the reference drops, land in b2_last_status().

namespace {

// Whole KV blocks of `block_bytes` between `cache` and the end of the device allocation that
// holds it (0 when unknown). The reference's run_decode_attn does not pass the pool size; the
// allocation's extent bounds it, which lets the kernel stage blocks with TMA (a tensor map
// needs the pool's extent) and check block-table entries against it.
int pool_blocks_of(const void* cache, size_t block_bytes) {
    typedef CUresult (*RangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);
    static RangeFn fn = nullptr;
    static bool resolved = false;
    static std::mutex mu;
    {
        std::lock_guard<std::mutex> lk(mu);
        if (!resolved) {
            void* ptr = nullptr;
            cudaDriverEntryPointQueryResult q;
            if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
                q == cudaDriverEntryPointSuccess)
                fn = reinterpret_cast<RangeFn>(ptr);
            resolved = true;
        }
    }
    if (!fn || !cache || block_bytes == 0) return 0;
    CUdeviceptr base = 0;
    size_t size = 0;
    if (fn(&base, &size, (CUdeviceptr)(uintptr_t)cache) != CUDA_SUCCESS) {
        cudaGetLastError();
        return 0;
    }
    const size_t avail = (size_t)(base + size - (CUdeviceptr)(uintptr_t)cache);
    return (int)std::min<size_t>(avail / block_bytes, 0x7fffffff);
}

}  // namespace

void run_decode_attn(int B, int H_q, int H_kv, int d, const float* Q, const float* k_cache, const float* v_cache,
                     const int* block_table, const int* context_lens, int max_context_len, int block_size,
                     int num_blocks_per_seq, float* O, float* workspace) {
    b2_decode_attn_args a{};
    a.B = B; a.H_q = H_q; a.H_kv = H_kv; a.head_dim = d;
    a.Q = Q; a.k_cache = k_cache; a.v_cache = v_cache; a.kv_dtype = B2_KV_F32;
    a.block_table = block_table; a.context_lens = context_lens;
    a.max_context_len = max_context_len; a.block_size = block_size; a.num_blocks_per_seq = num_blocks_per_seq;
    const size_t block_bytes = (size_t)(block_size > 0 ? block_size : 0) * (H_kv > 0 ? H_kv : 0) * (d > 0 ? d : 0) * 4;
    a.num_phys_blocks = std::min(pool_blocks_of(k_cache, block_bytes), pool_blocks_of(v_cache, block_bytes));
    a.scale = 0.f; a.O = O;
    a.workspace = workspace;
    a.workspace_bytes = (size_t)(B > 0 ? B : 0) * (H_q > 0 ? H_q : 0) * DA_MAX_SPLITS * (d + 2) * sizeof(float);
    t_last_status = decode_attn_launch(&a, false, 0);
}

void run_quantize_fp32_to_int8(int rows, int cols, const float* input, int32_t* output_packed, float* scales) {
    t_last_status = quantize_launch(rows, cols, input, output_packed, scales, 0);
}

void run_int8_gemm(int M, int N, int K, const int32_t* A_packed, const int32_t* BT_packed, const float* scale_A,
                   const float* scale_B, float* C) {
    t_last_status = gemm_launch(M, N, K, A_packed, BT_packed, scale_A, scale_B, nullptr, nullptr, C, B2_EPI_PLAIN,
                                false, 0);
}

void run_int8_gemm_bias(int M, int N, int K, const int32_t* A_packed, const int32_t* BT_packed,
                        const float* scale_A, const float* scale_B, const float* bias, float* C) {
    t_last_status = gemm_launch(M, N, K, A_packed, BT_packed, scale_A, scale_B, bias, nullptr, C, B2_EPI_BIAS, false, 0);
}

void run_int8_gemm_bias_gelu(int M, int N, int K, const int32_t* A_packed, const int32_t* BT_packed,
                             const float* scale_A, const float* scale_B, const float* bias, float* C) {
    t_last_status =
        gemm_launch(M, N, K, A_packed, BT_packed, scale_A, scale_B, bias, nullptr, C, B2_EPI_BIAS_GELU, false, 0);
}

void run_int8_gemm_bias_residual(int M, int N, int K, const int32_t* A_packed, const int32_t* BT_packed,
                                 const float* scale_A, const float* scale_B, const float* bias,
                                 const float* residual, float* C) {
    t_last_status = gemm_launch(M, N, K, A_packed, BT_packed, scale_A, scale_B, bias, residual, C,
                                B2_EPI_BIAS_RESIDUAL, false, 0);
}
