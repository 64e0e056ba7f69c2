// Batched GPT-2 INT8 decode engine (include/b2engine.h): weights, paged KV pool, block
// allocator, the decode step as a fixed launch sequence, and its CUDA-graph replay.
#include "common.cuh"
#include "tp_collectives.cuh"
#include "engine_kernels.cuh"
#include "b2engine.h"
#include <cuda_bf16.h>
#include <nccl.h>
#include "nccl_bounded.h"
#include <dlfcn.h>
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <numeric>
#include <random>
#include <string>
#include <vector>
#include <mutex>
#include <sys/stat.h>

namespace b2 {

int decode_attn_launch(const b2_decode_attn_args* a, bool counters_zeroed, cudaStream_t st);
int decode_attn_launch_ex(const b2_decode_attn_args* a, bool counters_zeroed, bool kv_early, cudaStream_t st);
// Decode attention reads the caches' older blocks before waiting on the QKV GEMM (on unless
// B2_ATTN_KV_EARLY=0).
static bool kv_early_on() {
    static const bool off = getenv("B2_ATTN_KV_EARLY") && strcmp(getenv("B2_ATTN_KV_EARLY"), "0") == 0;
    return !off;
}
size_t decode_attn_workspace_size(int B, int H_q, int H_kv, int D, int max_ctx, int block_size);
int quantize_launch(int rows, int cols, const float* in, int32_t* out, float* scales, cudaStream_t st);
int gemm_launch(int M, int N, int K, const int32_t* A, const int32_t* BT, const float* sA, const float* sB,
                const float* bias, const float* residual, void* C, int epi, bool s32, cudaStream_t st,
                void* ws = nullptr, size_t ws_bytes = 0);
size_t gemm_workspace_size(int M, int N, int K);
size_t gemm_rs_workspace_size(int M, int N, int K);

// NCCL is resolved at run time, only when tensor parallelism is used, preferring a
// libnccl.so.2 the process already loaded (e.g. PyTorch's), so loading this library never
// forces a second NCCL version into a process.
struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
    ncclResult_t (*GetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
    bool ok = false;
};

const NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
        api.AllReduce = reinterpret_cast<decltype(api.AllReduce)>(dlsym(h, "ncclAllReduce"));
        api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(dlsym(h, "ncclCommDestroy"));
        api.AllGather = reinterpret_cast<decltype(api.AllGather)>(dlsym(h, "ncclAllGather"));
        api.CommInitRankConfig =
            reinterpret_cast<decltype(api.CommInitRankConfig)>(dlsym(h, "ncclCommInitRankConfig"));
        api.GetAsyncError = reinterpret_cast<decltype(api.GetAsyncError)>(dlsym(h, "ncclCommGetAsyncError"));
        api.CommAbort = reinterpret_cast<decltype(api.CommAbort)>(dlsym(h, "ncclCommAbort"));
        api.CommFinalize = reinterpret_cast<decltype(api.CommFinalize)>(dlsym(h, "ncclCommFinalize"));
        api.ok = api.GetUniqueId && api.AllReduce && api.CommDestroy && api.AllGather &&
                 api.CommInitRankConfig && api.GetAsyncError && api.CommAbort && api.CommFinalize;
    });
    return api;
}

constexpr int kBlock = 16;        // KV block size (reference engine: block_size_ = 16)
constexpr int kPrefillRows = 8192;  // prompt tokens per prefill pass (longer prompts run in chunks)
constexpr int kPrefillItemRows = 16;  // rows of one sequence per prefill-attention CTA (PA_PQ)
constexpr int kCandCap = 256;     // argmax candidates recorded per row and step
constexpr float kLnEps = 1e-5f;   // reference LayerNorm eps (15_layernorm_residual.cuh default)

// Device linear layer in the reference's QuantWeight format + bias.
struct QLinear {
    int32_t* w = nullptr;  // [N, K/4]
    float* s = nullptr;    // [N]
    float* bias = nullptr; // [N]
    int N = 0, K = 0;
};

struct Layer {
    float *ln1_g = nullptr, *ln1_b = nullptr, *ln2_g = nullptr, *ln2_b = nullptr;
    QLinear qkv, out, up, down;
};

// Counter-based normal generator (SplitMix64 hash + Box-Muller), for seeded random weights.
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__global__ void randn_kernel(float* out, size_t n, uint64_t seed, float stddev) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const uint64_t r = mix64(seed * 0x100000001B3ull + i);
        const float u1 = ((uint32_t)(r >> 40) + 1u) * (1.0f / 16777217.0f);  // (0, 1]
        const float u2 = (uint32_t)(r & 0xFFFFFFu) * (1.0f / 16777216.0f);
        out[i] = stddev * sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
    }
}

__global__ void randn_bf16_kernel(__nv_bfloat16* out, size_t n, uint64_t seed) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const uint64_t r = mix64(seed * 0x100000001B3ull + i);
        const float u1 = ((uint32_t)(r >> 40) + 1u) * (1.0f / 16777217.0f);
        const float u2 = (uint32_t)(r & 0xFFFFFFu) * (1.0f / 16777216.0f);
        out[i] = __float2bfloat16_rn(sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2));
    }
}

__global__ void fill_kernel(float* out, size_t n, float v) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = v;
}

}  // namespace b2

using namespace b2;

struct b2_engine {
    b2_gpt2_config cfg{};
    int max_batch = 0, kv_dtype = B2_KV_F32;
    int device = 0;
    // tensor parallelism: this rank holds heads [rank*Hl, (rank+1)*Hl), i.e. model columns
    // [rank*dl, (rank+1)*dl), FFN columns [rank*ffl, ...) and vocab rows [v0, v0+Vl)
    int tp_rank = 0, tp_size = 1;
    int Hl = 0, dl = 0, ffl = 0, v0 = 0, Vl = 0;
    ncclComm_t comm = nullptr;
    // peer-memory collectives (tp_collectives.cu): every rank's x, acc32 and exchange region
    // mapped into this process; p2p = false falls back to NCCL all-reduces
    bool p2p = false;
    TpPeers peers{};
    unsigned char* xchg = nullptr;
    std::vector<void*> ipc_opened;
    float* amax = nullptr;    // [B] row absmax (row-parallel quantisation)
    int32_t* acc32 = nullptr; // [B, d] int32 partials of the row-parallel linears
    // exchange rows of the decode GEMMs whose K range is reduce-scattered over a cluster
    // (large activations: d_model or d_ff >= 2048 at batch 128)
    void* gemm_ws = nullptr;
    size_t gemm_ws_bytes = 0;
    std::vector<void*> allocs;  // every device allocation, freed by the destructor
    float *wte = nullptr, *wpe = nullptr, *lnf_g = nullptr, *lnf_b = nullptr;
    std::vector<Layer> layers;
    // paged KV pool: per layer [P, 16, H, d_head]
    int num_blocks = 0, blocks_per_seq = 0;
    void* k_pool = nullptr;
    void* v_pool = nullptr;
    size_t layer_stride = 0;  // elements per layer in a pool
    std::vector<int> free_blocks;
    // per-sequence state (device)
    int batch = 0, out_stride = 0;
    int *tokens = nullptr, *pos = nullptr, *ctx = nullptr, *block_table = nullptr;
    int *forced = nullptr, *forced_len = nullptr, *out_tokens = nullptr;
    int forced_stride = 0;
    unsigned long long* keys = nullptr;
    int* next_tok = nullptr;  // [max_batch] greedy token of the last step (b2_engine_decode_step)
    float rs_delta = 0.f;     // candidate margin of the exact argmax (twice the bf16x3 error bound)
    int* cand_cnt = nullptr;  // [max_batch] argmax candidates recorded by the vocab projection
    void* cand = nullptr;     // [max_batch, kCandCap] (value bits, local vocab index)
    // activations
    float *x = nullptr, *qkv = nullptr, *q = nullptr, *attn = nullptr, *hbuf = nullptr, *xf = nullptr;
    float* logits = nullptr;
    bool keep_logits = false;
    void *wte_hi = nullptr, *wte_lo = nullptr;  // bf16 halves of wte for the tensor-core vocab projection
    void *xf_hi = nullptr, *xf_lo = nullptr;    // bf16 halves of the final hidden state
    int32_t* xq = nullptr;
    float* xs = nullptr;
    void* attn_ws = nullptr;
    size_t attn_ws_bytes = 0;
    // CUDA graph of one step
    cudaGraphExec_t graph = nullptr;
    bool graph_dirty = true;
    bool failed = false;  // a device allocation failed
    // host copies of the current sequences' prompts and block tables (prefill builds its rows
    // from them); at_start: no step has run since b2_engine_start (every position is 0)
    std::vector<int> host_prompts, host_prompt_lens, host_bt;
    int host_prompt_stride = 0;
    bool at_start = false;
    // batched prefill: one row per prompt token, buffers allocated on first use for pf_cap rows
    int pf_cap = 0;
    int *pf_tokens = nullptr, *pf_pos = nullptr, *pf_ctx = nullptr, *pf_bt = nullptr;
    int2* pf_items = nullptr;
    unsigned long long* pf_keys = nullptr;
    float *pf_x = nullptr, *pf_qkv = nullptr, *pf_q = nullptr, *pf_attn = nullptr, *pf_hbuf = nullptr, *pf_xs = nullptr,
          *pf_amax = nullptr;
    int32_t *pf_xq = nullptr, *pf_acc32 = nullptr;
    void* pf_ws = nullptr;
    size_t pf_ws_bytes = 0;
    // exact fp32 argmax after the tensor-core projection (B2_EXACT_ARGMAX=0: the bf16x3 argmax)
    bool exact_argmax = !(getenv("B2_EXACT_ARGMAX") && strcmp(getenv("B2_EXACT_ARGMAX"), "0") == 0);
    // fused QKV split in the GEMM epilogue (B2_ENGINE_FUSE_QKV=0 runs GEMM + scatter kernel)
    bool fuse_qkv = !(getenv("B2_ENGINE_FUSE_QKV") && strcmp(getenv("B2_ENGINE_FUSE_QKV"), "0") == 0);

    ~b2_engine();
    template <typename T>
    T* alloc(size_t n) {
        void* p = nullptr;
        if (n == 0) n = 1;
        if (cudaMalloc(&p, n * sizeof(T)) != cudaSuccess) {
            failed = true;
            return nullptr;
        }
        allocs.push_back(p);
        return static_cast<T*>(p);
    }
};

b2_engine::~b2_engine() {
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(device);
    if (graph) cudaGraphExecDestroy(graph);
    cudaDeviceSynchronize();
    for (void* p : ipc_opened) cudaIpcCloseMemHandle(p);
    // peers tear down within moments of each other; a gone peer costs at most a minute here
    if (comm) comm_destroy_bounded(nccl(), comm, std::min(nccl_timeout_s(), 60.0));
    for (void* p : allocs) cudaFree(p);
    cudaSetDevice(cur);
}

namespace {

bool valid_config(const b2_gpt2_config& c) {
    return c.n_layers > 0 && c.n_heads > 0 && c.d_head > 0 && c.d_model == c.n_heads * c.d_head &&
           (c.d_head == 64 || c.d_head == 128) && c.d_ff > 0 && c.vocab_size > 0 && c.max_seq_len > 0 &&
           c.d_model % 16 == 0 && c.d_ff % 16 == 0 && c.d_model <= 8192;
}

// Device buffers that do not depend on the weights' source.
int alloc_runtime(b2_engine* e) {
    const b2_gpt2_config& c = e->cfg;
    const int B = e->max_batch, d = c.d_model;
    e->blocks_per_seq = (c.max_seq_len + kBlock - 1) / kBlock;
    e->num_blocks = B * e->blocks_per_seq;
    const size_t kvb = e->kv_dtype == B2_KV_F32 ? 4 : 2;
    e->layer_stride = (size_t)e->num_blocks * kBlock * e->dl;
    const size_t pool_bytes = (size_t)c.n_layers * e->layer_stride * kvb;
    e->k_pool = e->alloc<unsigned char>(pool_bytes);
    e->v_pool = e->alloc<unsigned char>(pool_bytes);
    e->tokens = e->alloc<int>(B);
    e->pos = e->alloc<int>(B);
    e->ctx = e->alloc<int>(B);
    e->block_table = e->alloc<int>((size_t)B * e->blocks_per_seq);
    e->keys = e->alloc<unsigned long long>(2 * (size_t)B);  // approximate, then exact argmax keys
    e->next_tok = e->alloc<int>(B);
    e->cand_cnt = e->alloc<int>(B);
    e->cand = e->alloc<int2>((size_t)B * kCandCap);
    e->x = e->alloc<float>((size_t)B * d);
    e->qkv = e->alloc<float>((size_t)B * 3 * e->dl);
    e->q = e->alloc<float>((size_t)B * d);
    e->attn = e->alloc<float>((size_t)B * d);
    e->hbuf = e->alloc<float>((size_t)B * e->ffl);
    e->amax = e->alloc<float>(B);
    e->acc32 = e->alloc<int32_t>((size_t)B * d);
    e->xf = e->alloc<float>((size_t)B * d);
    e->logits = e->alloc<float>((size_t)B * e->Vl);
    e->xq = e->alloc<int32_t>((size_t)B * std::max(d, c.d_ff) / 4);
    e->xs = e->alloc<float>(B);
    e->wte_hi = e->alloc<uint16_t>((size_t)e->Vl * d);
    e->wte_lo = e->alloc<uint16_t>((size_t)e->Vl * d);
    e->xf_hi = e->alloc<uint16_t>((size_t)B * d);
    e->xf_lo = e->alloc<uint16_t>((size_t)B * d);
    e->attn_ws_bytes = std::max<size_t>(256, decode_attn_workspace_size(B, e->Hl, e->Hl, c.d_head, c.max_seq_len,
                                                                         kBlock));
    e->attn_ws = e->alloc<unsigned char>(e->attn_ws_bytes);
    {
        const int kl = d / e->tp_size, kf = c.d_ff / e->tp_size;
        const size_t g = std::max({gemm_rs_workspace_size(B, 3 * e->dl, d), gemm_rs_workspace_size(B, d, kl),
                                   gemm_rs_workspace_size(B, e->ffl, d), gemm_rs_workspace_size(B, d, kf)});
        if (g) {
            e->gemm_ws = e->alloc<unsigned char>(g);
            e->gemm_ws_bytes = g;
        }
    }
    if (e->failed) return B2_ERR_CUDA;
    if (!e->k_pool || !e->v_pool || !e->attn_ws || !e->logits) return B2_ERR_CUDA;
    if (cudaMemset(e->attn_ws, 0, e->attn_ws_bytes) != cudaSuccess) return B2_ERR_CUDA;
    if (cudaMemset(e->cand_cnt, 0, (size_t)B * sizeof(int)) != cudaSuccess) return B2_ERR_CUDA;
    if (cudaMemset(e->k_pool, 0, pool_bytes) != cudaSuccess || cudaMemset(e->v_pool, 0, pool_bytes) != cudaSuccess)
        return B2_ERR_CUDA;
    e->free_blocks.resize(e->num_blocks);
    std::iota(e->free_blocks.begin(), e->free_blocks.end(), 0);
    return B2_OK;
}

int alloc_weights(b2_engine* e) {
    const b2_gpt2_config& c = e->cfg;
    const int d = c.d_model;
    e->wte = e->alloc<float>((size_t)c.vocab_size * d);
    e->wpe = e->alloc<float>((size_t)c.max_seq_len * d);
    e->lnf_g = e->alloc<float>(d);
    e->lnf_b = e->alloc<float>(d);
    e->layers.resize(c.n_layers);
    auto lin = [&](QLinear& L, int N, int K) {
        L.N = N;
        L.K = K;
        L.w = e->alloc<int32_t>((size_t)N * K / 4);
        L.s = e->alloc<float>(N);
        L.bias = e->alloc<float>(N);
        return L.w && L.s && L.bias;
    };
    for (Layer& l : e->layers) {
        l.ln1_g = e->alloc<float>(d);
        l.ln1_b = e->alloc<float>(d);
        l.ln2_g = e->alloc<float>(d);
        l.ln2_b = e->alloc<float>(d);
        if (!lin(l.qkv, 3 * e->dl, d) || !lin(l.out, d, e->dl) || !lin(l.up, e->ffl, d) || !lin(l.down, d, e->ffl))
            return B2_ERR_CUDA;
        if (!l.ln1_g || !l.ln1_b || !l.ln2_g || !l.ln2_b) return B2_ERR_CUDA;
    }
    return (e->wte && e->wpe && e->lnf_g && e->lnf_b) ? B2_OK : B2_ERR_CUDA;
}

void randn(float* p, size_t n, uint64_t seed, float sd) { randn_kernel<<<1184, 256>>>(p, n, seed, sd); }
void fill(float* p, size_t n, float v) { fill_kernel<<<592, 256>>>(p, n, v); }

// fp32 [N, K] weight drawn N(0, 0.02), then quantised per row in place of the reference's
// offline exporter (python/export_gpt2.py:10-40, same arithmetic as the GPU quantiser).
int random_linear(QLinear& L, uint64_t seed, float* tmp) {
    randn(tmp, (size_t)L.N * L.K, seed, 0.02f);
    int st = quantize_launch(L.N, L.K, tmp, L.w, L.s, 0);
    if (st != B2_OK) return st;
    randn(L.bias, L.N, seed ^ 0xB1A5ull, 0.02f);
    return B2_OK;
}

// ---- reference on-disk format (src/gpt2_engine.cu:19-112, python/export_gpt2.py:59-187)
bool read_file(const std::string& path, void* host, size_t bytes) {
    std::ifstream f(path, std::ios::binary);
    if (!f) return false;
    f.read(static_cast<char*>(host), (std::streamsize)bytes);
    return (size_t)f.gcount() == bytes;  // a short file is an error (the reference does not check)
}
bool load_dev(const std::string& path, void* dev, size_t bytes) {
    std::vector<char> h(bytes);
    if (!read_file(path, h.data(), bytes)) return false;
    return cudaMemcpy(dev, h.data(), bytes, cudaMemcpyHostToDevice) == cudaSuccess;
}
bool write_file(const std::string& path, const void* host, size_t bytes) {
    std::ofstream f(path, std::ios::binary);
    if (!f) return false;
    f.write(static_cast<const char*>(host), (std::streamsize)bytes);
    return (bool)f;
}
bool save_dev(const std::string& path, const void* dev, size_t bytes) {
    std::vector<char> h(bytes);
    if (cudaMemcpy(h.data(), dev, bytes, cudaMemcpyDeviceToHost) != cudaSuccess) return false;
    return write_file(path, h.data(), bytes);
}

// config.json with the reference's seven integer keys (parse: find key, atoi after ':').
bool parse_config(const std::string& path, b2_gpt2_config& c) {
    std::ifstream f(path);
    if (!f) return false;
    std::string s((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    auto get = [&](const char* key, int& out) {
        size_t p = s.find(std::string("\"") + key + "\"");
        if (p == std::string::npos) return false;
        p = s.find(':', p);
        if (p == std::string::npos) return false;
        out = atoi(s.c_str() + p + 1);
        return true;
    };
    return get("n_layers", c.n_layers) && get("n_heads", c.n_heads) && get("d_model", c.d_model) &&
           get("d_ff", c.d_ff) && get("vocab_size", c.vocab_size) && get("max_seq_len", c.max_seq_len) &&
           get("d_head", c.d_head);
}

int mkdir_p(const std::string& dir) {
    for (size_t i = 1; i <= dir.size(); ++i) {
        if (i == dir.size() || dir[i] == '/') {
            const std::string sub = dir.substr(0, i);
            struct stat sb;
            if (stat(sub.c_str(), &sb) != 0 && mkdir(sub.c_str(), 0755) != 0) return -1;
        }
    }
    return 0;
}

std::string layer_dir(const std::string& root, int i) {
    char buf[32];
    snprintf(buf, sizeof(buf), "/layer_%02d", i);
    return root + buf;
}

}  // namespace

namespace {

// One decode step: a fixed sequence of launches on `st` (capturable as a CUDA graph).
// Enables programmatic dependent launch for the launches of one decode step: every kernel in
// the step reads only constant weights before its griddep_wait().
struct PdlScope : PdlOn {
    PdlScope() : PdlOn(/*constant_weights=*/true) {}
};

// Optional per-launch timing of one eager step: an event is recorded on the step's stream
// before every launch (and after the last), and the intervals are summed per label. The
// events serialise the launches (no programmatic overlap), so the report is a breakdown of
// where a step goes, not a faster or slower step.
struct StepProfiler {
    cudaStream_t st = nullptr;
    std::vector<std::pair<const char*, cudaEvent_t>> marks;
    bool ok = true;
    void mark(const char* label) {
        cudaEvent_t ev = nullptr;
        if (cudaEventCreate(&ev) != cudaSuccess || cudaEventRecord(ev, st) != cudaSuccess) ok = false;
        marks.push_back({label, ev});
    }
    ~StepProfiler() {
        for (auto& m : marks)
            if (m.second) cudaEventDestroy(m.second);
    }
};

// The rows one pass of the layer stack runs over: the decode step's batch (one row per
// sequence, at its current position) or a prefill chunk (one row per prompt token). Every
// row carries its token, position, context length (position + 1, written by the embedding)
// and block-table row; activations and workspaces are sized for n rows.
struct RowSet {
    int n = 0;
    const int* tokens = nullptr;
    const int* pos = nullptr;
    int* ctx = nullptr;
    const int* block_table = nullptr;  // [n, blocks_per_seq]
    unsigned long long* keys = nullptr;
    float *x = nullptr, *qkv = nullptr, *q = nullptr, *attn = nullptr, *hbuf = nullptr, *xs = nullptr, *amax = nullptr;
    int32_t *xq = nullptr, *acc32 = nullptr;
    void* attn_ws = nullptr;
    size_t attn_ws_bytes = 0;
    void* gemm_ws = nullptr;  // reduce-scatter exchange rows (decode rows only)
    size_t gemm_ws_bytes = 0;
    int max_ctx = 0;
    bool p2p = false;  // the peer-memory exchange (its buffers are the decode step's)
    // prefill: causal attention over work items (first row, rows) of one sequence each
    const int2* items = nullptr;
    int n_items = 0;
};

// Embedding and every transformer layer for the rows of R (no final LayerNorm / vocab).
int enqueue_layers(b2_engine* e, const RowSet& R, cudaStream_t st, StepProfiler* prof) {
    auto M = [&](const char* label) {
        if (prof) prof->mark(label);
    };
    const b2_gpt2_config& c = e->cfg;
    const int B = R.n, d = c.d_model, ff = c.d_ff, dh = c.d_head;
    const size_t kvb = e->kv_dtype == B2_KV_F32 ? 4 : 2;
    int r;
#define B2_TRY(x) do { if ((r = (x)) != B2_OK) return r; } while (0)
    M("embed");
    B2_TRY(launch_embed(B, d, R.tokens, R.pos, e->wte, e->wpe, R.x, R.ctx, R.keys, st));
    const bool tp = e->tp_size > 1;
    const int Hl = e->Hl, dl = e->dl, ffl = e->ffl;
    // the exchange rows go only to GEMMs that take the reduce-scatter split: a workspace
    // given to another shape would select the global-memory split-K path instead
    auto gws = [&](int N, int K) { return gemm_rs_workspace_size(B, N, K) ? R.gemm_ws : nullptr; };
    auto gwb = [&](int N, int K) { return gemm_rs_workspace_size(B, N, K) && R.gemm_ws ? R.gemm_ws_bytes : 0; };
    // all-reduces of the tensor-parallel step (NCCL on the step's stream; captured in the graph)
    auto allreduce = [&](void* buf, size_t n, ncclDataType_t t, ncclRedOp_t op) {
        return nccl_call_bounded(nccl(), e->comm, [&] { return nccl().AllReduce(buf, buf, n, t, op, e->comm, st); },
                                 nccl_timeout_s());
    };
    // row-parallel linear: global-scale quantisation of this rank's activation columns,
    // local int32 GEMM over them, int32 all-reduce (exact), then the dequant epilogue
    auto row_parallel = [&](const float* act, int kl, const QLinear& W, const char* gemm_label) {
        int r2;
        if (R.p2p) {
            M("tp_quantize");
            if ((r2 = launch_tp_quantize(B, kl, act, R.xq, R.xs, e->peers, st)) != B2_OK) return r2;
            M(gemm_label);
            if ((r2 = gemm_launch(B, d, kl, R.xq, W.w, nullptr, nullptr, nullptr, nullptr, R.acc32, B2_EPI_PLAIN,
                                  true, st, gws(d, kl), gwb(d, kl))) != B2_OK)
                return r2;
            M("tp_reduce");
            return launch_tp_reduce(B, d, R.xs, W.s, W.bias, e->peers, st);
        }
        M("rowmax");
        if ((r2 = launch_rowmax(B, kl, act, R.amax, st)) != B2_OK) return r2;
        M("allreduce_amax");
        if ((r2 = allreduce(R.amax, B, ncclFloat, ncclMax)) != B2_OK) return r2;
        M("quantize_scaled");
        if ((r2 = launch_quantize_scaled(B, kl, act, R.amax, R.xq, R.xs, st)) != B2_OK) return r2;
        M(gemm_label);
        if ((r2 = gemm_launch(B, d, kl, R.xq, W.w, nullptr, nullptr, nullptr, nullptr, R.acc32, B2_EPI_PLAIN, true,
                              st, gws(d, kl), gwb(d, kl))) != B2_OK)
            return r2;
        M("allreduce_partials");
        if ((r2 = allreduce(R.acc32, (size_t)B * d, ncclInt32, ncclSum)) != B2_OK) return r2;
        M("dequant_residual");
        return launch_dequant_residual(B, d, R.acc32, R.xs, W.s, W.bias, R.x, R.x, st);
    };
    for (int l = 0; l < c.n_layers; ++l) {
        const Layer& L = e->layers[l];
        unsigned char* kc = static_cast<unsigned char*>(e->k_pool) + (size_t)l * e->layer_stride * kvb;
        unsigned char* vc = static_cast<unsigned char*>(e->v_pool) + (size_t)l * e->layer_stride * kvb;
        // attention sub-block (pre-norm; x stays the residual and is updated in place)
        M("ln_quant");
        B2_TRY(launch_ln_quant(B, d, R.x, L.ln1_g, L.ln1_b, kLnEps, R.xq, R.xs, nullptr, st));
        // QKV linear with the split into q and the paged K/V write in its epilogue; shapes the
        // fused path does not take run as GEMM + scatter kernel
        M("gemm_qkv");
        QkvScatterArgs qa;
        qa.q = R.q;
        qa.k = kc;
        qa.v = vc;
        qa.pos = R.pos;
        qa.block_table = R.block_table;
        qa.d = dl;
        qa.block_size = kBlock;
        qa.nbps = e->blocks_per_seq;
        qa.bf16 = e->kv_dtype == B2_KV_BF16;
        r = e->fuse_qkv ? gemm_launch_qkv(B, 3 * dl, d, R.xq, L.qkv.w, R.xs, L.qkv.s, L.qkv.bias, qa, st,
                                          gws(3 * dl, d), gwb(3 * dl, d))
                        : B2_ERR_UNSUPPORTED;
        if (r == B2_ERR_UNSUPPORTED) {
            B2_TRY(gemm_launch(B, 3 * dl, d, R.xq, L.qkv.w, R.xs, L.qkv.s, L.qkv.bias, nullptr, R.qkv, B2_EPI_BIAS,
                               false, st, gws(3 * dl, d), gwb(3 * dl, d)));
            M("qkv_scatter");
            B2_TRY(launch_qkv_scatter(B, dl, Hl, dh, kBlock, e->blocks_per_seq, R.qkv, R.pos, R.block_table, R.q, kc,
                                      vc, e->kv_dtype, st));
        } else if (r != B2_OK) {
            return r;
        }
        b2_decode_attn_args a{};
        a.B = B; a.H_q = Hl; a.H_kv = Hl; a.head_dim = dh;
        a.Q = R.q; a.k_cache = kc; a.v_cache = vc; a.kv_dtype = e->kv_dtype;
        a.block_table = R.block_table; a.context_lens = R.ctx;
        a.max_context_len = R.max_ctx; a.block_size = kBlock; a.num_blocks_per_seq = e->blocks_per_seq;
        a.num_phys_blocks = e->num_blocks; a.scale = 0.f; a.O = R.attn;
        a.workspace = R.attn_ws; a.workspace_bytes = R.attn_ws_bytes;
        M("attention");
        if (R.items)
            B2_TRY(launch_prefill_attention(R.items, R.n_items, Hl, dh, e->kv_dtype, R.q, kc, vc, R.block_table,
                                            e->blocks_per_seq, kBlock, R.pos, R.attn, st));
        else  // the caches' older blocks, table and lengths predate the QKV GEMM before this launch
            B2_TRY(decode_attn_launch_ex(&a, true, kv_early_on(), st));
        if (tp) {
            B2_TRY(row_parallel(R.attn, dl, L.out, "gemm_out"));
        } else {
            M("quantize");
            B2_TRY(quantize_launch(B, d, R.attn, R.xq, R.xs, st));
            M("gemm_out");
            B2_TRY(gemm_launch(B, d, d, R.xq, L.out.w, R.xs, L.out.s, L.out.bias, R.x, R.x, B2_EPI_BIAS_RESIDUAL,
                               false, st, gws(d, d), gwb(d, d)));
        }
        // MLP sub-block
        M("ln_quant");
        B2_TRY(launch_ln_quant(B, d, R.x, L.ln2_g, L.ln2_b, kLnEps, R.xq, R.xs, nullptr, st));
        M("gemm_fc1");
        B2_TRY(gemm_launch(B, ffl, d, R.xq, L.up.w, R.xs, L.up.s, L.up.bias, nullptr, R.hbuf, B2_EPI_BIAS_GELU, false,
                           st, gws(ffl, d), gwb(ffl, d)));
        if (tp) {
            B2_TRY(row_parallel(R.hbuf, ffl, L.down, "gemm_fc2"));
        } else {
            M("quantize");
            B2_TRY(quantize_launch(B, ff, R.hbuf, R.xq, R.xs, st));
            M("gemm_fc2");
            B2_TRY(gemm_launch(B, d, ff, R.xq, L.down.w, R.xs, L.down.s, L.down.bias, R.x, R.x, B2_EPI_BIAS_RESIDUAL,
                               false, st, gws(d, ff), gwb(d, ff)));
        }
    }
#undef B2_TRY
    return B2_OK;
}

int enqueue_step(b2_engine* e, cudaStream_t st, StepProfiler* prof = nullptr) {
    PdlScope pdl;
    auto M = [&](const char* label) {
        if (prof) prof->mark(label);
    };
    const b2_gpt2_config& c = e->cfg;
    const int B = e->batch, d = c.d_model;
    const bool tp = e->tp_size > 1;
    RowSet R;
    R.n = B;
    R.tokens = e->tokens;
    R.pos = e->pos;
    R.ctx = e->ctx;
    R.block_table = e->block_table;
    R.keys = e->keys;
    R.x = e->x; R.qkv = e->qkv; R.q = e->q; R.attn = e->attn; R.hbuf = e->hbuf; R.xs = e->xs; R.amax = e->amax;
    R.xq = e->xq; R.acc32 = e->acc32;
    R.attn_ws = e->attn_ws;
    R.attn_ws_bytes = e->attn_ws_bytes;
    R.gemm_ws = e->gemm_ws;
    R.gemm_ws_bytes = e->gemm_ws_bytes;
    R.max_ctx = c.max_seq_len;
    R.p2p = e->p2p;
    int r;
#define B2_TRY(x) do { if ((r = (x)) != B2_OK) return r; } while (0)
    B2_TRY(enqueue_layers(e, R, st, prof));
    auto allreduce = [&](void* buf, size_t n, ncclDataType_t t, ncclRedOp_t op) {
        return nccl_call_bounded(nccl(), e->comm, [&] { return nccl().AllReduce(buf, buf, n, t, op, e->comm, st); },
                                 nccl_timeout_s());
    };
    M("ln_final");
    B2_TRY(launch_ln_quant(B, d, e->x, e->lnf_g, e->lnf_b, kLnEps, nullptr, nullptr, e->xf, st, e->xf_hi,
                           e->xf_lo));
    M("vocab_argmax");
    float* logits = e->keep_logits ? e->logits : nullptr;
    B2_TRY((launch_vocab_bf16x3(B, e->Vl, d, e->xf_hi, e->xf_lo, e->wte_hi, e->wte_lo, logits, e->keys, st, e->v0,
                               e->rs_delta, e->exact_argmax ? e->cand_cnt : nullptr,
                               e->exact_argmax ? e->cand : nullptr, kCandCap)));
    // exact fp32 value of every argmax candidate (this rank's vocab rows), so the greedy token
    // is the one the reference's fp32 projection picks
    unsigned long long* keys_exact = e->keys;
    if (e->exact_argmax) {
        M("vocab_rescore");
        keys_exact = e->keys + B;
        B2_TRY(launch_vocab_rescore(B, e->Vl, d, e->v0, e->xf, e->wte, e->rs_delta, logits, e->keys, keys_exact,
                                    e->cand_cnt, e->cand, kCandCap, st));
    }
    if (tp) {
        M("allreduce_keys");
        B2_TRY(allreduce(keys_exact, B, ncclUint64, ncclMax));  // global argmax over the vocab shards
    }
    M("advance");
    B2_TRY(launch_advance(B, keys_exact, e->tokens, e->pos, e->forced, e->forced_len, e->forced_stride, e->out_tokens,
                          e->out_stride, c.max_seq_len, st, e->next_tok));
#undef B2_TRY
    return B2_OK;
}

// Maps every rank's x, acc32 and exchange region into this process for the peer-memory
// collectives: CUDA IPC handles all-gathered over the engine's NCCL communicator. Every rank
// runs the same collectives whatever happens locally, and all ranks agree (all-reduce min)
// before switching p2p on, so a failure on one rank leaves every rank on NCCL all-reduces.
// The closing all-reduce is also the barrier after which peers may write into this rank's
// zeroed exchange region. B2_TP_COLLECTIVES=nccl keeps the NCCL path.
// A rank whose allocations failed (local_ok false) still takes part, so no rank is left
// waiting in a collective.
int setup_peers(b2_engine* e, bool local_ok) {
    const int world = e->tp_size, rank = e->tp_rank;
    const char* env = getenv("B2_TP_COLLECTIVES");
    if (!e->comm || world < 2 || world > TP_MAX_RANKS || (env && strcmp(env, "nccl") == 0)) return B2_OK;
    const TpLayout L = TpLayout::make(e->max_batch);
    e->xchg = local_ok ? e->alloc<unsigned char>(L.bytes) : nullptr;
    struct Blob {
        cudaIpcMemHandle_t h[3];
        int ok;
        int pad[15];
    };
    Blob mine{};
    mine.ok = local_ok && e->xchg && (e->cfg.d_model % 4) == 0 && cudaMemset(e->xchg, 0, L.bytes) == cudaSuccess &&
              cudaIpcGetMemHandle(&mine.h[0], e->x) == cudaSuccess &&
              cudaIpcGetMemHandle(&mine.h[1], e->acc32) == cudaSuccess &&
              cudaIpcGetMemHandle(&mine.h[2], e->xchg) == cudaSuccess;
    unsigned char* dbuf = nullptr;
    if (cudaDeviceSynchronize() != cudaSuccess || cudaMalloc(&dbuf, (size_t)(world + 1) * sizeof(Blob) + 16) != cudaSuccess)
        return B2_ERR_CUDA;
    std::vector<Blob> all(world);
    int agreed = 0;
    bool nccl_ok = cudaMemcpy(dbuf, &mine, sizeof(Blob), cudaMemcpyHostToDevice) == cudaSuccess &&
                   nccl_call_bounded(nccl(), e->comm, [&] {
                       return nccl().AllGather(dbuf, dbuf + sizeof(Blob), sizeof(Blob), ncclUint8, e->comm, 0);
                   }, nccl_timeout_s()) == B2_OK &&
                   cudaMemcpy(all.data(), dbuf + sizeof(Blob), world * sizeof(Blob), cudaMemcpyDeviceToHost) ==
                       cudaSuccess;
    TpPeers P{};
    int opened = nccl_ok ? 1 : 0;
    for (int p = 0; p < world; ++p) opened = opened && all[p].ok;
    for (int p = 0; opened && p < world; ++p) {
        if (p == rank) {
            P.x[p] = e->x;
            P.acc[p] = e->acc32;
            P.xchg[p] = e->xchg;
            continue;
        }
        void* ptr[3] = {nullptr, nullptr, nullptr};
        for (int k = 0; k < 3 && opened; ++k) {
            if (cudaIpcOpenMemHandle(&ptr[k], all[p].h[k], cudaIpcMemLazyEnablePeerAccess) == cudaSuccess)
                e->ipc_opened.push_back(ptr[k]);
            else
                opened = 0;
        }
        P.x[p] = static_cast<float*>(ptr[0]);
        P.acc[p] = static_cast<const int32_t*>(ptr[1]);
        P.xchg[p] = static_cast<unsigned char*>(ptr[2]);
    }
    int* flag = reinterpret_cast<int*>(dbuf + (size_t)(world + 1) * sizeof(Blob));
    nccl_ok = nccl_ok && cudaMemcpy(flag, &opened, sizeof(int), cudaMemcpyHostToDevice) == cudaSuccess &&
              nccl_call_bounded(nccl(), e->comm, [&] {
                  return nccl().AllReduce(flag, flag, 1, ncclInt32, ncclMin, e->comm, 0);
              }, nccl_timeout_s()) == B2_OK &&
              cudaMemcpy(&agreed, flag, sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess;
    cudaFree(dbuf);
    if (!nccl_ok) return B2_ERR_CUDA;
    if (!agreed) {
        for (void* p : e->ipc_opened) cudaIpcCloseMemHandle(p);
        e->ipc_opened.clear();
        return B2_OK;
    }
    P.L = L;
    P.rank = rank;
    P.world = world;
    P.err = device_error_ptr();
    e->peers = P;
    e->p2p = true;
    return B2_OK;
}

int finish_create(b2_engine* e, b2_engine** out) {
    // bf16 hi/lo halves of the tied embedding for the tensor-core vocab projection
    if (launch_split_bf16(e->wte + (size_t)e->v0 * e->cfg.d_model, e->wte_hi, e->wte_lo,
                          (size_t)e->Vl * e->cfg.d_model, 0) != B2_OK ||
        cudaDeviceSynchronize() != cudaSuccess) {
        delete e;
        return B2_ERR_CUDA;
    }
    // margin of the exact argmax: 2 * 2^-10 * max ||h|| * max ||wte_v||, with the final
    // LayerNorm's output bounded by ||h|| <= max|gamma| sqrt(d) + ||beta|| (its normalised row
    // has norm sqrt(d) at most; 1.001 covers the rounding)
    const int d = e->cfg.d_model;
    const float wmax = row_norm_max(e->Vl, d, e->wte + (size_t)e->v0 * d);
    std::vector<float> g(d), bt(d);
    if (!(wmax >= 0.f) || cudaMemcpy(g.data(), e->lnf_g, d * 4, cudaMemcpyDeviceToHost) != cudaSuccess ||
        cudaMemcpy(bt.data(), e->lnf_b, d * 4, cudaMemcpyDeviceToHost) != cudaSuccess) {
        delete e;
        return B2_ERR_CUDA;
    }
    double gmax = 0.0, bn = 0.0;
    for (int i = 0; i < d; ++i) {
        gmax = std::max(gmax, (double)std::fabs(g[i]));
        bn += (double)bt[i] * bt[i];
    }
    const double hmax = 1.001 * gmax * std::sqrt((double)d) + std::sqrt(bn);
    e->rs_delta = (float)(2.0 * std::ldexp(1.0, -10) * hmax * wmax);
    *out = e;
    return B2_OK;
}

}  // namespace

namespace {

int set_tp(b2_engine* e, int rank, int world) {
    const b2_gpt2_config& c = e->cfg;
    if (c.n_heads % world || c.d_ff % world || ((c.d_ff / world) % 16) || ((c.n_heads / world * c.d_head) % 16))
        return B2_ERR_UNSUPPORTED;
    e->tp_rank = rank;
    e->tp_size = world;
    e->Hl = c.n_heads / world;
    e->dl = e->Hl * c.d_head;
    e->ffl = c.d_ff / world;
    const int per = (c.vocab_size + world - 1) / world;
    e->v0 = std::min(c.vocab_size, rank * per);
    e->Vl = std::max(1, std::min(per, c.vocab_size - e->v0));
    return B2_OK;
}

// Copies this rank's slice of a full linear: rows [r0, r0+rows) of each of `segs` equal
// row segments (column-parallel), or every row's K columns [k0, k0+kl) (row-parallel).
int copy_rows(QLinear& dst, const QLinear& full, int segs, int rows, int rank) {
    const int seg_rows = full.N / segs;
    const size_t kb = (size_t)full.K;  // int8 bytes per row
    for (int s = 0; s < segs; ++s) {
        const size_t src_row = (size_t)s * seg_rows + (size_t)rank * rows, dst_row = (size_t)s * rows;
        if (cudaMemcpy(reinterpret_cast<char*>(dst.w) + dst_row * kb, reinterpret_cast<const char*>(full.w) + src_row * kb,
                       rows * kb, cudaMemcpyDeviceToDevice) != cudaSuccess ||
            cudaMemcpy(dst.s + dst_row, full.s + src_row, rows * 4, cudaMemcpyDeviceToDevice) != cudaSuccess ||
            cudaMemcpy(dst.bias + dst_row, full.bias + src_row, rows * 4, cudaMemcpyDeviceToDevice) != cudaSuccess)
            return B2_ERR_CUDA;
    }
    return B2_OK;
}
int copy_cols(QLinear& dst, const QLinear& full, int kl, int rank) {
    if (cudaMemcpy2D(dst.w, kl, reinterpret_cast<const char*>(full.w) + (size_t)rank * kl, full.K, kl, full.N,
                     cudaMemcpyDeviceToDevice) != cudaSuccess ||
        cudaMemcpy(dst.s, full.s, (size_t)full.N * 4, cudaMemcpyDeviceToDevice) != cudaSuccess ||
        cudaMemcpy(dst.bias, full.bias, (size_t)full.N * 4, cudaMemcpyDeviceToDevice) != cudaSuccess)
        return B2_ERR_CUDA;
    return B2_OK;
}

int create_random_impl(const b2_gpt2_config* cfg, int max_batch, int kv_dtype, uint64_t seed, int rank, int world,
                       const void* nccl_id, b2_engine** out) {
    if (!cfg || !out || max_batch <= 0 || !valid_config(*cfg)) return B2_ERR_INVALID;
    if (kv_dtype != B2_KV_F32 && kv_dtype != B2_KV_BF16) return B2_ERR_UNSUPPORTED;
    b2_engine* e = new b2_engine();
    e->cfg = *cfg;
    e->max_batch = max_batch;
    e->kv_dtype = kv_dtype;
    cudaGetDevice(&e->device);
    int st = set_tp(e, rank, world);
    if (st == B2_OK && world > 1) {
        ncclUniqueId id;
        memcpy(&id, nccl_id, sizeof(id));
        // non-blocking creation with a bound: a rank that never joins is a timeout, not a hang
        st = nccl().ok ? comm_init_bounded(nccl(), &e->comm, world, id, rank, nccl_timeout_s()) : B2_ERR_CUDA;
    }
    if (st == B2_OK) st = alloc_weights(e);
    if (st == B2_OK) st = alloc_runtime(e);
    if (e->comm) {
        const int sp = setup_peers(e, st == B2_OK);
        if (st == B2_OK) st = sp;
    }
    if (st != B2_OK) {
        delete e;
        return st;
    }
    const b2_gpt2_config& c = e->cfg;
    const int d = c.d_model, ff = c.d_ff;
    // every rank draws the full weights with the 1-GPU seeds and keeps its slice, so a
    // tensor-parallel engine computes the same model as the unsharded one
    const size_t maxNK = (size_t)std::max(3 * d, ff) * std::max(d, ff);
    float* tmp = nullptr;
    QLinear full;
    bool ok = cudaMalloc(&tmp, maxNK * 4) == cudaSuccess && cudaMalloc(&full.w, maxNK) == cudaSuccess &&
              cudaMalloc(&full.s, (size_t)std::max(3 * d, ff) * 4) == cudaSuccess &&
              cudaMalloc(&full.bias, (size_t)std::max(3 * d, ff) * 4) == cudaSuccess;
    randn(e->wte, (size_t)c.vocab_size * d, seed * 16 + 1, 0.02f);
    randn(e->wpe, (size_t)c.max_seq_len * d, seed * 16 + 2, 0.02f);
    fill(e->lnf_g, d, 1.f);
    fill(e->lnf_b, d, 0.f);
    for (int l = 0; ok && l < c.n_layers; ++l) {
        Layer& L = e->layers[l];
        fill(L.ln1_g, d, 1.f);
        fill(L.ln1_b, d, 0.f);
        fill(L.ln2_g, d, 1.f);
        fill(L.ln2_b, d, 0.f);
        const uint64_t sd = seed * 1000003ull + 97ull * (l + 1);
        full.N = 3 * d; full.K = d;
        ok = ok && random_linear(full, sd + 1, tmp) == B2_OK && copy_rows(L.qkv, full, 3, e->dl, rank) == B2_OK;
        full.N = d; full.K = d;
        ok = ok && random_linear(full, sd + 2, tmp) == B2_OK && copy_cols(L.out, full, e->dl, rank) == B2_OK;
        full.N = ff; full.K = d;
        ok = ok && random_linear(full, sd + 3, tmp) == B2_OK && copy_rows(L.up, full, 1, e->ffl, rank) == B2_OK;
        full.N = d; full.K = ff;
        ok = ok && random_linear(full, sd + 4, tmp) == B2_OK && copy_cols(L.down, full, e->ffl, rank) == B2_OK;
    }
    cudaDeviceSynchronize();
    cudaFree(tmp);
    cudaFree(full.w);
    cudaFree(full.s);
    cudaFree(full.bias);
    if (!ok) {
        delete e;
        return B2_ERR_CUDA;
    }
    return finish_create(e, out);
}

}  // namespace

// ------------------------------------------------------------------ C ABI
extern "C" {

int b2_engine_create_random(const b2_gpt2_config* cfg, int max_batch, int kv_dtype, uint64_t seed, b2_engine** out) {
    return create_random_impl(cfg, max_batch, kv_dtype, seed, 0, 1, nullptr, out);
}

int b2_nccl_unique_id(void* out, size_t bytes) {
    if (!out || bytes < sizeof(ncclUniqueId)) return B2_ERR_INVALID;
    ncclUniqueId id;
    if (!nccl().ok || nccl().GetUniqueId(&id) != ncclSuccess) return B2_ERR_CUDA;
    memcpy(out, &id, sizeof(id));
    return B2_OK;
}

int b2_engine_create_random_tp(const b2_gpt2_config* cfg, int max_batch, int kv_dtype, uint64_t seed,
                               const void* nccl_id, int rank, int world, b2_engine** out) {
    if (!nccl_id || world < 1 || rank < 0 || rank >= world) return B2_ERR_INVALID;
    return create_random_impl(cfg, max_batch, kv_dtype, seed, rank, world, nccl_id, out);
}

int b2_engine_load(const char* model_dir, int max_batch, int kv_dtype, b2_engine** out) {
    if (!model_dir || !out || max_batch <= 0) return B2_ERR_INVALID;
    if (kv_dtype != B2_KV_F32 && kv_dtype != B2_KV_BF16) return B2_ERR_UNSUPPORTED;
    b2_gpt2_config c{};
    const std::string root(model_dir);
    if (!parse_config(root + "/config.json", c) || !valid_config(c)) return B2_ERR_INVALID;
    b2_engine* e = new b2_engine();
    e->cfg = c;
    e->max_batch = max_batch;
    e->kv_dtype = kv_dtype;
    cudaGetDevice(&e->device);
    int st = set_tp(e, 0, 1);
    if (st == B2_OK) st = alloc_weights(e);
    if (st == B2_OK) st = alloc_runtime(e);
    const int d = c.d_model;
    bool ok = st == B2_OK;
    auto f32 = [&](const std::string& path, float* dev, size_t n) { ok = ok && load_dev(path, dev, n * 4); };
    auto qlin = [&](const std::string& dir, const char* name, QLinear& L) {
        ok = ok && load_dev(dir + "/" + name + "_weight.bin", L.w, (size_t)L.N * L.K) &&
             load_dev(dir + "/" + name + "_scale.bin", L.s, (size_t)L.N * 4) &&
             load_dev(dir + "/" + name + "_bias.bin", L.bias, (size_t)L.N * 4);
    };
    f32(root + "/wte.bin", e->wte, (size_t)c.vocab_size * d);
    f32(root + "/wpe.bin", e->wpe, (size_t)c.max_seq_len * d);
    f32(root + "/ln_f_gamma.bin", e->lnf_g, d);
    f32(root + "/ln_f_beta.bin", e->lnf_b, d);
    for (int l = 0; ok && l < c.n_layers; ++l) {
        const std::string ld = layer_dir(root, l);
        Layer& L = e->layers[l];
        f32(ld + "/ln1_gamma.bin", L.ln1_g, d);
        f32(ld + "/ln1_beta.bin", L.ln1_b, d);
        f32(ld + "/ln2_gamma.bin", L.ln2_g, d);
        f32(ld + "/ln2_beta.bin", L.ln2_b, d);
        qlin(ld, "qkv", L.qkv);
        qlin(ld, "out", L.out);
        qlin(ld, "ffn_up", L.up);
        qlin(ld, "ffn_down", L.down);
    }
    if (!ok) {
        delete e;
        return st != B2_OK ? st : B2_ERR_INVALID;
    }
    return finish_create(e, out);
}

int b2_engine_export(const b2_engine* e, const char* model_dir) {
    if (!e || !model_dir) return B2_ERR_INVALID;
    if (e->tp_size != 1) return B2_ERR_UNSUPPORTED;  // a rank holds only its shard
    const b2_gpt2_config& c = e->cfg;
    const std::string root(model_dir);
    char js[512];
    snprintf(js, sizeof(js),
             "{\n  \"n_layers\": %d,\n  \"n_heads\": %d,\n  \"d_model\": %d,\n  \"d_ff\": %d,\n  \"vocab_size\": %d,\n"
             "  \"max_seq_len\": %d,\n  \"d_head\": %d\n}\n",
             c.n_layers, c.n_heads, c.d_model, c.d_ff, c.vocab_size, c.max_seq_len, c.d_head);
    bool ok = mkdir_p(root) == 0 && write_file(root + "/config.json", js, strlen(js));
    const int d = c.d_model;
    auto f32 = [&](const std::string& path, const float* dev, size_t n) { ok = ok && save_dev(path, dev, n * 4); };
    auto qlin = [&](const std::string& dir, const char* name, const QLinear& L) {
        ok = ok && save_dev(dir + "/" + name + "_weight.bin", L.w, (size_t)L.N * L.K) &&
             save_dev(dir + "/" + name + "_scale.bin", L.s, (size_t)L.N * 4) &&
             save_dev(dir + "/" + name + "_bias.bin", L.bias, (size_t)L.N * 4);
    };
    f32(root + "/wte.bin", e->wte, (size_t)c.vocab_size * d);
    f32(root + "/wpe.bin", e->wpe, (size_t)c.max_seq_len * d);
    f32(root + "/ln_f_gamma.bin", e->lnf_g, d);
    f32(root + "/ln_f_beta.bin", e->lnf_b, d);
    for (int l = 0; ok && l < c.n_layers; ++l) {
        const std::string ld = layer_dir(root, l);
        if (mkdir_p(ld) != 0) return B2_ERR_INVALID;
        const Layer& L = e->layers[l];
        f32(ld + "/ln1_gamma.bin", L.ln1_g, d);
        f32(ld + "/ln1_beta.bin", L.ln1_b, d);
        f32(ld + "/ln2_gamma.bin", L.ln2_g, d);
        f32(ld + "/ln2_beta.bin", L.ln2_b, d);
        qlin(ld, "qkv", L.qkv);
        qlin(ld, "out", L.out);
        qlin(ld, "ffn_up", L.up);
        qlin(ld, "ffn_down", L.down);
    }
    return ok ? B2_OK : B2_ERR_INVALID;
}

void b2_engine_destroy(b2_engine* e) { delete e; }

int b2_engine_config(const b2_engine* e, b2_gpt2_config* out) {
    if (!e || !out) return B2_ERR_INVALID;
    *out = e->cfg;
    return B2_OK;
}

int b2_engine_start(b2_engine* e, int batch, const int32_t* prompts_host, const int32_t* prompt_lens_host,
                    int prompt_stride, int max_new_tokens, uint64_t seed) {
    if (!e || !prompts_host || !prompt_lens_host || batch <= 0 || batch > e->max_batch || max_new_tokens < 0 ||
        prompt_stride <= 0)
        return B2_ERR_INVALID;
    const b2_gpt2_config& c = e->cfg;
    int max_total = 0;
    for (int b = 0; b < batch; ++b) {
        const int pl = prompt_lens_host[b];
        if (pl < 1 || pl > prompt_stride || pl + max_new_tokens > c.max_seq_len) return B2_ERR_INVALID;
        for (int i = 0; i < pl; ++i)
            if (prompts_host[(size_t)b * prompt_stride + i] < 0 || prompts_host[(size_t)b * prompt_stride + i] >= c.vocab_size)
                return B2_ERR_INVALID;
        max_total = std::max(max_total, pl + max_new_tokens);
    }
    // block allocator: return every block to the free list and hand each sequence the blocks
    // it can ever need. seed 0: in pool order, as the reference engine allocates
    // (src/gpt2_engine.cu:420-429, physical block = logical block); any other seed shuffles
    // the free list first, so block tables are scattered over the whole pool
    e->free_blocks.resize(e->num_blocks);
    std::iota(e->free_blocks.rbegin(), e->free_blocks.rend(), 0);  // popped from the back: 0, 1, 2, ...
    if (seed != 0) {
        std::mt19937_64 rng(seed);
        std::shuffle(e->free_blocks.begin(), e->free_blocks.end(), rng);
    }
    std::vector<int> bt((size_t)batch * e->blocks_per_seq, 0);
    for (int b = 0; b < batch; ++b) {
        // every sequence owns blocks for the whole max_seq_len, so a step past the requested
        // length can never touch another sequence's blocks
        const int need = e->blocks_per_seq;
        if ((int)e->free_blocks.size() < need) return B2_ERR_INVALID;
        for (int j = 0; j < need; ++j) {
            bt[(size_t)b * e->blocks_per_seq + j] = e->free_blocks.back();
            e->free_blocks.pop_back();
        }
    }
    // forced (prompt) tokens and the output record live in one allocation per start
    const int stride = prompt_stride;
    const int ostride = max_total + 1;
    if (!e->forced || e->forced_stride < stride || e->batch < batch || e->out_stride < ostride) {
        e->forced = e->alloc<int>((size_t)e->max_batch * stride);
        e->forced_len = e->alloc<int>(e->max_batch);
        e->out_tokens = e->alloc<int>((size_t)e->max_batch * ostride);
        if (e->failed) return B2_ERR_CUDA;
    }
    e->forced_stride = stride;
    e->out_stride = ostride;
    e->batch = batch;
    std::vector<int> tok(batch), zero(batch, 0);
    for (int b = 0; b < batch; ++b) tok[b] = prompts_host[(size_t)b * stride];
    bool ok = cudaMemcpy(e->block_table, bt.data(), bt.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
              cudaMemcpy(e->forced, prompts_host, (size_t)batch * stride * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
              cudaMemcpy(e->forced_len, prompt_lens_host, (size_t)batch * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
              cudaMemcpy(e->tokens, tok.data(), (size_t)batch * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
              cudaMemcpy(e->pos, zero.data(), (size_t)batch * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
              cudaMemset(e->out_tokens, 0xff, (size_t)batch * ostride * 4) == cudaSuccess;
    e->graph_dirty = true;  // the batch size or buffers may have changed
    e->host_prompts.assign(prompts_host, prompts_host + (size_t)batch * stride);
    e->host_prompt_lens.assign(prompt_lens_host, prompt_lens_host + batch);
    e->host_prompt_stride = stride;
    e->host_bt = bt;
    e->at_start = ok;
    return ok ? B2_OK : B2_ERR_CUDA;
}

int b2_engine_step(b2_engine* e, b2_stream_t stream) {
    if (!e || e->batch <= 0) return B2_ERR_INVALID;
    e->at_start = false;
    return enqueue_step(e, static_cast<cudaStream_t>(stream));
}

int b2_engine_prefill(b2_engine* e, b2_stream_t stream) {
    if (!e || e->batch <= 0 || !e->at_start) return B2_ERR_INVALID;
    const b2_gpt2_config& c = e->cfg;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int nbps = e->blocks_per_seq;
    // rows: every prompt token but each sequence's last, in (sequence, position) order
    std::vector<int> rb, rp;
    for (int b = 0; b < e->batch; ++b)
        for (int p = 0; p + 1 < e->host_prompt_lens[b]; ++p) {
            rb.push_back(b);
            rp.push_back(p);
        }
    const int total = (int)rb.size();
    if (total > 0 && e->pf_cap == 0) {
        const int cap = std::min(total, kPrefillRows);
        const int d = c.d_model;
        e->pf_tokens = e->alloc<int>(cap);
        e->pf_pos = e->alloc<int>(cap);
        e->pf_ctx = e->alloc<int>(cap);
        e->pf_bt = e->alloc<int>((size_t)cap * nbps);
        e->pf_items = e->alloc<int2>(cap);
        e->pf_keys = e->alloc<unsigned long long>(2 * (size_t)cap);
        e->pf_x = e->alloc<float>((size_t)cap * d);
        e->pf_qkv = e->alloc<float>((size_t)cap * 3 * e->dl);
        e->pf_q = e->alloc<float>((size_t)cap * d);
        e->pf_attn = e->alloc<float>((size_t)cap * d);
        e->pf_hbuf = e->alloc<float>((size_t)cap * e->ffl);
        e->pf_xs = e->alloc<float>(cap);
        e->pf_amax = e->alloc<float>(cap);
        e->pf_xq = e->alloc<int32_t>((size_t)cap * std::max(d, c.d_ff) / 4);
        e->pf_acc32 = e->alloc<int32_t>((size_t)cap * d);
        e->pf_ws_bytes = std::max<size_t>(256, decode_attn_workspace_size(cap, e->Hl, e->Hl, c.d_head, c.max_seq_len,
                                                                          kBlock));
        e->pf_ws = e->alloc<unsigned char>(e->pf_ws_bytes);
        if (e->failed || cudaMemset(e->pf_ws, 0, e->pf_ws_bytes) != cudaSuccess) return B2_ERR_CUDA;
        e->pf_cap = cap;
    }
    std::vector<int> tok, pos, bt;
    std::vector<int2> items;
    for (int r0 = 0; r0 < total; r0 += e->pf_cap) {
        const int n = std::min(e->pf_cap, total - r0);
        tok.resize(n);
        pos.resize(n);
        bt.resize((size_t)n * nbps);
        items.clear();
        int max_ctx = 1;
        for (int i = 0; i < n; ++i) {
            const int b = rb[r0 + i], p = rp[r0 + i];
            tok[i] = e->host_prompts[(size_t)b * e->host_prompt_stride + p];
            pos[i] = p;
            max_ctx = std::max(max_ctx, p + 1);
            std::copy(e->host_bt.begin() + (size_t)b * nbps, e->host_bt.begin() + (size_t)(b + 1) * nbps,
                      bt.begin() + (size_t)i * nbps);
            // attention work items: runs of up to kPrefillItemRows rows of one sequence
            if (items.empty() || rb[r0 + items.back().x] != b || items.back().y == kPrefillItemRows)
                items.push_back(make_int2(i, 1));
            else
                ++items.back().y;
        }
        // the previous chunk has finished with the row arrays before they are overwritten
        if (cudaStreamSynchronize(st) != cudaSuccess ||
            cudaMemcpy(e->pf_tokens, tok.data(), (size_t)n * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(e->pf_pos, pos.data(), (size_t)n * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(e->pf_bt, bt.data(), bt.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(e->pf_items, items.data(), items.size() * sizeof(int2), cudaMemcpyHostToDevice) != cudaSuccess)
            return B2_ERR_CUDA;
        RowSet R;
        R.n = n;
        R.tokens = e->pf_tokens;
        R.pos = e->pf_pos;
        R.ctx = e->pf_ctx;
        R.block_table = e->pf_bt;
        R.keys = e->pf_keys;
        R.x = e->pf_x; R.qkv = e->pf_qkv; R.q = e->pf_q; R.attn = e->pf_attn; R.hbuf = e->pf_hbuf; R.xs = e->pf_xs;
        R.amax = e->pf_amax; R.xq = e->pf_xq; R.acc32 = e->pf_acc32;
        R.attn_ws = e->pf_ws;
        R.attn_ws_bytes = e->pf_ws_bytes;
        R.max_ctx = max_ctx;
        R.p2p = false;  // the peer-mapped buffers are the decode step's: NCCL all-reduces here
        R.items = e->pf_items;
        R.n_items = (int)items.size();
        PdlScope pdl;
        const int r = enqueue_layers(e, R, st, nullptr);
        if (r != B2_OK) return r;
    }
    // continue at each sequence's last prompt token: the next step feeds it and predicts the
    // first new token, exactly as after prompt_len - 1 steps
    std::vector<int> tok_last(e->batch), pos_last(e->batch);
    for (int b = 0; b < e->batch; ++b) {
        pos_last[b] = e->host_prompt_lens[b] - 1;
        tok_last[b] = e->host_prompts[(size_t)b * e->host_prompt_stride + pos_last[b]];
    }
    if (cudaStreamSynchronize(st) != cudaSuccess ||
        cudaMemcpy(e->tokens, tok_last.data(), (size_t)e->batch * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(e->pos, pos_last.data(), (size_t)e->batch * 4, cudaMemcpyHostToDevice) != cudaSuccess)
        return B2_ERR_CUDA;
    e->at_start = false;
    return B2_OK;
}

int b2_engine_profile_step(b2_engine* e, char* report, size_t report_bytes) {
    if (!e || e->batch <= 0 || !report || report_bytes == 0) return B2_ERR_INVALID;
    e->at_start = false;
    cudaStream_t st;
    if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess) return B2_ERR_CUDA;
    int r = B2_OK;
    {
        StepProfiler prof;
        prof.st = st;
        r = enqueue_step(e, st, &prof);
        prof.mark("end");
        if (cudaStreamSynchronize(st) != cudaSuccess || !prof.ok) r = B2_ERR_CUDA;
        if (r == B2_OK) {
            struct Agg {
                const char* label;
                int n;
                double us;
            };
            std::vector<Agg> agg;
            for (size_t i = 0; i + 1 < prof.marks.size(); ++i) {
                float ms = 0.f;
                cudaEventElapsedTime(&ms, prof.marks[i].second, prof.marks[i + 1].second);
                auto it = std::find_if(agg.begin(), agg.end(),
                                       [&](const Agg& a) { return strcmp(a.label, prof.marks[i].first) == 0; });
                if (it == agg.end()) {
                    agg.push_back({prof.marks[i].first, 0, 0.0});
                    it = agg.end() - 1;
                }
                it->n += 1;
                it->us += ms * 1e3;
            }
            float total_ms = 0.f;
            cudaEventElapsedTime(&total_ms, prof.marks.front().second, prof.marks.back().second);
            std::sort(agg.begin(), agg.end(), [](const Agg& a, const Agg& b) { return a.us > b.us; });
            std::string out;
            char line[160];
            snprintf(line, sizeof(line), "step_us %.1f launches %zu\n", total_ms * 1e3, prof.marks.size() - 1);
            out += line;
            for (const Agg& a : agg) {
                snprintf(line, sizeof(line), "%-20s %5d %10.1f %6.1f%%\n", a.label, a.n, a.us,
                         total_ms > 0.f ? 100.0 * a.us / (total_ms * 1e3) : 0.0);
                out += line;
            }
            snprintf(report, report_bytes, "%s", out.c_str());
        }
    }
    cudaStreamDestroy(st);
    return r;
}

int b2_engine_run_steps(b2_engine* e, int steps, b2_stream_t stream) {
    if (!e || e->batch <= 0 || steps < 0) return B2_ERR_INVALID;
    if (steps > 0) e->at_start = false;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (e->graph_dirty || !e->graph) {
        if (e->graph) {
            cudaGraphExecDestroy(e->graph);
            e->graph = nullptr;
        }
        // capture on a private stream so the caller's stream may be the legacy default one
        cudaStream_t cap;
        if (cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking) != cudaSuccess) return B2_ERR_CUDA;
        cudaGraph_t g = nullptr;
        int r = B2_OK;
        if (cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal) != cudaSuccess) r = B2_ERR_CUDA;
        if (r == B2_OK) r = enqueue_step(e, cap);
        if (cudaStreamEndCapture(cap, &g) != cudaSuccess && r == B2_OK) r = B2_ERR_CUDA;
        if (r == B2_OK && cudaGraphInstantiate(&e->graph, g, 0) != cudaSuccess) r = B2_ERR_CUDA;
        if (g) cudaGraphDestroy(g);
        cudaStreamDestroy(cap);
        if (r != B2_OK) return r;
        e->graph_dirty = false;
    }
    for (int i = 0; i < steps; ++i)
        if (cudaGraphLaunch(e->graph, st) != cudaSuccess) return B2_ERR_CUDA;
    return B2_OK;
}

int b2_engine_decode_step(b2_engine* e, const int32_t* tokens_in, int32_t* next_out, b2_stream_t stream) {
    if (!e || e->batch <= 0 || !tokens_in) return B2_ERR_INVALID;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const size_t n = (size_t)e->batch * sizeof(int32_t);
    // the caller's tokens replace whatever the previous step (or the prompt) left as input
    if (cudaMemcpyAsync(e->tokens, tokens_in, n, cudaMemcpyDefault, st) != cudaSuccess) return B2_ERR_CUDA;
    const int r = b2_engine_run_steps(e, 1, stream);
    if (r != B2_OK) return r;
    if (next_out && cudaMemcpyAsync(next_out, e->next_tok, n, cudaMemcpyDefault, st) != cudaSuccess)
        return B2_ERR_CUDA;
    return B2_OK;
}

int b2_engine_read_tokens(const b2_engine* e, int32_t* out_host, int out_stride) {
    if (!e || !out_host || e->batch <= 0 || out_stride <= 0) return B2_ERR_INVALID;
    std::vector<int> buf((size_t)e->batch * e->out_stride);
    if (cudaMemcpy(buf.data(), e->out_tokens, buf.size() * 4, cudaMemcpyDeviceToHost) != cudaSuccess) return B2_ERR_CUDA;
    for (int b = 0; b < e->batch; ++b)
        for (int p = 0; p < out_stride; ++p)
            out_host[(size_t)b * out_stride + p] = p < e->out_stride ? buf[(size_t)b * e->out_stride + p] : -1;
    return B2_OK;
}

int b2_engine_keep_logits(b2_engine* e, int enable, const float** logits) {
    if (!e) return B2_ERR_INVALID;
    if (e->keep_logits != (enable != 0)) e->graph_dirty = true;
    e->keep_logits = enable != 0;
    if (logits) *logits = e->keep_logits ? e->logits : nullptr;
    return B2_OK;
}

int b2_engine_read_logits(const b2_engine* e, float* out_host) {
    if (!e || !out_host || e->batch <= 0 || !e->keep_logits) return B2_ERR_INVALID;
    return cudaMemcpy(out_host, e->logits, (size_t)e->batch * e->Vl * 4, cudaMemcpyDeviceToHost) ==
                   cudaSuccess
               ? B2_OK
               : B2_ERR_CUDA;
}

int b2_engine_fill_kv_random(b2_engine* e, int ctx_len, uint64_t seed) {
    if (e) e->at_start = false;
    if (!e || e->batch <= 0 || ctx_len < 0 || ctx_len >= e->cfg.max_seq_len) return B2_ERR_INVALID;
    const size_t n = (size_t)e->cfg.n_layers * e->layer_stride;
    for (int which = 0; which < 2; ++which) {
        void* pool = which ? e->v_pool : e->k_pool;
        const uint64_t sd = seed * 4 + which + 2ull * e->tp_rank * 0x9E37ull;
        if (e->kv_dtype == B2_KV_F32)
            randn_kernel<<<1184, 256>>>(static_cast<float*>(pool), n, sd, 1.0f);
        else
            randn_bf16_kernel<<<1184, 256>>>(static_cast<__nv_bfloat16*>(pool), n, sd);
    }
    std::vector<int> p(e->batch, ctx_len);
    if (cudaMemcpy(e->pos, p.data(), (size_t)e->batch * 4, cudaMemcpyHostToDevice) != cudaSuccess) return B2_ERR_CUDA;
    return cudaDeviceSynchronize() == cudaSuccess ? B2_OK : B2_ERR_CUDA;
}

int b2_engine_positions(const b2_engine* e, int32_t* pos_host) {
    if (!e || !pos_host || e->batch <= 0) return B2_ERR_INVALID;
    return cudaMemcpy(pos_host, e->pos, (size_t)e->batch * 4, cudaMemcpyDeviceToHost) == cudaSuccess ? B2_OK
                                                                                                       : B2_ERR_CUDA;
}

}  // extern "C"
