// Host side of the decode engine: GGUF loading and weight repacking, the
// encoder pass, the fixed-buffer greedy step and its CUDA-graph cache, and the
// C ABI of include/malaga_b200.h.
//
// Reference structure mirrored here (crates/malaga-core/src/):
//   model.rs:343-433   Nllb::load         -> Engine::load
//   model.rs:463-500   encode_cross       -> mgb_encode
//   graph.rs:23-135    StaticState        -> StaticState
//   graph.rs:138-140   bucket()           -> bucket()
//   graph.rs:173-334   GraphCache         -> Engine::greedy + the LRU cache
//   model.rs:552-612   step_static        -> Engine::launch_step
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <set>
#include <string>
#include <unordered_set>
#include <vector>

#include "../../include/malaga_b200.h"
#include "beam.cuh"
#include "gemm_tc.cuh"
#include "smallmm.cuh"
#include "stepkernel.cuh"

using namespace mgb;

// ---------------------------------------------------------------------------
// Errors

static thread_local std::string g_err;

static mgb_status set_err(mgb_status s, const char *fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    return s;
}

void mgb_internal_set_error(const char *msg) { g_err = msg; }

static mgb_status cuda_err(cudaError_t e, const char *what) {
    if (e == cudaErrorMemoryAllocation)
        return set_err(MGB_ERR_OOM, "%s: CUDA_ERROR_OUT_OF_MEMORY (%s)", what, cudaGetErrorString(e));
    return set_err(MGB_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

#define CK(call)                                                  \
    do {                                                          \
        cudaError_t e_ = (call);                                  \
        if (e_ != cudaSuccess) return cuda_err(e_, #call);        \
    } while (0)

#define TRY(call)                           \
    do {                                    \
        mgb_status s_ = (call);             \
        if (s_ != MGB_OK) return s_;        \
    } while (0)

// ---------------------------------------------------------------------------
// GGUF

namespace {

struct GgufTensor {
    std::string name;
    int type = -1;
    std::vector<uint64_t> dims;  // GGML order: dims[0] innermost
    const uint8_t *data = nullptr;
    long rows() const {
        long r = 1;
        for (size_t i = 1; i < dims.size(); ++i) r *= (long)dims[i];
        return r;
    }
    long cols() const { return dims.empty() ? 0 : (long)dims[0]; }
};

struct GgufFile {
    void *map = MAP_FAILED;
    size_t size = 0;
    std::map<std::string, uint64_t> u32;
    std::map<std::string, std::vector<uint32_t>> u32arr;  // arrays of u32 / i32 (shortlists)
    std::map<std::string, GgufTensor> tensors;
    ~GgufFile() {
        if (map != MAP_FAILED) munmap(map, size);
    }
};

long row_bytes(int type, long n) {
    switch (type) {
        case T_F32: return 4 * n;
        case T_F16: return 2 * n;
        case T_Q8_0: return n % 32 ? -1 : n / 32 * 34;
        case T_Q4_K: return n % 256 ? -1 : n / 256 * 144;
        case T_Q6_K: return n % 256 ? -1 : n / 256 * 210;
    }
    return -1;
}

mgb_status parse_gguf(const char *path, GgufFile &f) {
    int fd = open(path, O_RDONLY);
    if (fd < 0) return set_err(MGB_ERR_IO, "cannot open %s", path);
    struct stat st;
    fstat(fd, &st);
    f.size = (size_t)st.st_size;
    f.map = mmap(nullptr, f.size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (f.map == MAP_FAILED) return set_err(MGB_ERR_IO, "cannot map %s", path);
    const uint8_t *base = (const uint8_t *)f.map, *p = base, *end = base + f.size;
    auto need = [&](size_t n) { return (size_t)(end - p) >= n; };
    auto r32 = [&]() { uint32_t v; memcpy(&v, p, 4); p += 4; return v; };
    auto r64 = [&]() { uint64_t v; memcpy(&v, p, 8); p += 8; return v; };
    auto rstr = [&](std::string &s) -> bool {
        if (!need(8)) return false;
        uint64_t n = r64();
        if (!need(n)) return false;
        s.assign((const char *)p, n);
        p += n;
        return true;
    };
    if (!need(24) || r32() != 0x46554747u) return set_err(MGB_ERR_IO, "%s is not a GGUF file", path);
    uint32_t version = r32();
    if (version < 2) return set_err(MGB_ERR_IO, "unsupported GGUF version %u", version);
    uint64_t nt = r64(), nkv = r64();
    uint64_t align = 32;
    static const int scalar[] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
    std::function<bool(uint32_t)> skip = [&](uint32_t t) -> bool {
        if (t == 8) { std::string s; return rstr(s); }
        if (t == 9) {
            if (!need(12)) return false;
            uint32_t et = r32();
            uint64_t n = r64();
            for (uint64_t i = 0; i < n; ++i)
                if (!skip(et)) return false;
            return true;
        }
        if (t > 12 || !need(scalar[t])) return false;
        p += scalar[t];
        return true;
    };
    for (uint64_t i = 0; i < nkv; ++i) {
        std::string key;
        if (!rstr(key) || !need(4)) return set_err(MGB_ERR_IO, "truncated GGUF metadata");
        uint32_t t = r32();
        if (t == 4 || t == 5) {
            if (!need(4)) return set_err(MGB_ERR_IO, "truncated GGUF metadata");
            f.u32[key] = r32();
        } else if (t == 7 || t == 0 || t == 1) {
            if (!need(1)) return set_err(MGB_ERR_IO, "truncated GGUF metadata");
            f.u32[key] = *p++;
        } else if (t == 10 || t == 11) {
            if (!need(8)) return set_err(MGB_ERR_IO, "truncated GGUF metadata");
            f.u32[key] = r64();
        } else if (t == 9 && need(12) && (((const uint32_t *)p)[0] == 4 || ((const uint32_t *)p)[0] == 5)) {
            r32();
            const uint64_t n = r64();
            if (n > (uint64_t)(end - p) / 4) return set_err(MGB_ERR_IO, "truncated GGUF metadata");
            std::vector<uint32_t> &v = f.u32arr[key];
            v.resize(n);
            memcpy(v.data(), p, 4 * n);
            p += 4 * n;
        } else if (!skip(t)) {
            return set_err(MGB_ERR_IO, "bad GGUF metadata value for %s", key.c_str());
        }
    }
    if (f.u32.count("general.alignment")) align = f.u32["general.alignment"];
    std::vector<std::pair<std::string, uint64_t>> offs;
    for (uint64_t i = 0; i < nt; ++i) {
        GgufTensor t;
        if (!rstr(t.name) || !need(4)) return set_err(MGB_ERR_IO, "truncated GGUF tensor info");
        uint32_t nd = r32();
        if (nd < 1 || nd > 4 || !need(8 * nd + 12)) return set_err(MGB_ERR_IO, "bad tensor info %s", t.name.c_str());
        for (uint32_t k = 0; k < nd; ++k) t.dims.push_back(r64());
        t.type = (int)r32();
        offs.emplace_back(t.name, r64());
        f.tensors[t.name] = t;
    }
    size_t data0 = ((size_t)(p - base) + align - 1) / align * align;
    for (auto &o : offs) {
        GgufTensor &t = f.tensors[o.first];
        long rb = row_bytes(t.type, t.cols());
        if (rb < 0) return set_err(MGB_ERR_UNSUPPORTED, "tensor %s: type %d with rows of %ld values", t.name.c_str(), t.type, t.cols());
        if (data0 + o.second + (size_t)rb * t.rows() > f.size) return set_err(MGB_ERR_IO, "tensor %s past end of file", t.name.c_str());
        t.data = base + data0 + o.second;
    }
    return MGB_OK;
}

// Unpacks the 32 values of 32-block `j` of a Q4_K row (0..15) / Q6_K row (0..63).
void q4k_block_values(const uint8_t *row, int j, uint8_t *q) {
    const uint8_t *sb = row + (j / 8) * 144, *qs = sb + 16;
    const int i = j % 8, c = i / 2, hi = i & 1;
    for (int k = 0; k < 32; ++k) q[k] = hi ? (qs[32 * c + k] >> 4) : (qs[32 * c + k] & 0xf);
}

void q6k_block_values(const uint8_t *row, int j, uint8_t *q) {
    const uint8_t *b = row + (j / 8) * 210;
    for (int k = 0; k < 32; ++k) {
        const int i = (j % 8) * 32 + k, n = i / 128, g = (i % 128) / 32, l = i % 32;
        const uint8_t *ql = b + 64 * n, *qh = b + 128 + 32 * n;
        int v;
        switch (g) {
            case 0: v = (ql[l] & 0xf) | (((qh[l] >> 0) & 3) << 4); break;
            case 1: v = (ql[l + 32] & 0xf) | (((qh[l] >> 2) & 3) << 4); break;
            case 2: v = (ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4); break;
            default: v = (ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4); break;
        }
        q[k] = (uint8_t)v;
    }
}

}  // namespace

// ---------------------------------------------------------------------------
// Engine

// Split-K buffers of a decode step (StaticState): partials and tile counters.
struct SplitBufs {
    float2 *part = nullptr;
    uint32_t *count = nullptr;
    size_t part_units = 0;
};

struct StaticState {
    int b = 0, s = 0, m = 0;
    uint32_t *ids = nullptr, *step = nullptr, *out = nullptr, *lens = nullptr;
    uint8_t *finished = nullptr;
    float *x = nullptr, *q = nullptr, *a = nullptr, *u = nullptr, *xf = nullptr;
    QAct act;                        // q8_1 tensor-core activations of the next matmul
    QAct act2;                       // the FFN hidden rows' (written by the FFN-up epilogue)
    SplitBufs split;                 // split-K partials and tile counters
    // persistent step kernel (batches of at most 8 rows): its phase table, grid
    // barrier / abort words and shared-memory geometry
    StepPhase *phases = nullptr;
    int nphases = 0;
    uint32_t *bar = nullptr;
    unsigned long long *trace = nullptr;  // phase timing (MGB_STEP_TRACE)
    std::vector<StepPhase> phase_host;
    std::string trace_path;
    // --fast-vocab (shortlist index >= 0): the rows' source ids [b][s] (pad past
    // each row's length) and the best source-token logit of each 8 positions
    int sl = -1;
    uint32_t *src_ids = nullptr;
    float *src_emb = nullptr;  // their embedding rows, f32 [b][s][d]
    float *src_v = nullptr;
    uint32_t *src_i = nullptr;
    int step_slots = 0, step_slot_bytes = 0, step_act_bytes = 0, step_ctas = 0;
    size_t step_smem = 0;
    // beam search (allocated on first use): step logits, top-k, row sources, and
    // the generic decode's f32 caches (model.rs:124-133: self K/V, with a second
    // set to gather into; the sentences' cross K/V per beam row)
    float *beam_logits = nullptr, *beam_vals = nullptr;
    uint32_t *beam_idx = nullptr;
    int *beam_from = nullptr;
    std::vector<float *> kc32, vc32, kc32b, vc32b, ck32, cv32;
    std::vector<__half *> kc, vc, ck, cv;
    float *part_v = nullptr;
    uint32_t *part_i = nullptr;
    int lm_parts = 0;  // CTAs of the LM-head launch = argmax partials per row
    float *logits = nullptr;
    cudaGraphExec_t exec = nullptr;
    size_t graph_nodes = 0;
    size_t bytes = 0;
    uint64_t last_used = 0;
    std::vector<void *> allocs;
};

struct mgb_batch {
    int b = 0, s = 0;
    std::vector<uint32_t> lens;
    uint32_t *d_lens = nullptr;
    float *cross = nullptr;  // f32 [L][2][b][H][s][hd], as encode_cross returns it (model.rs:463-477)
    size_t cross_bytes = 0;
    void *buf = nullptr;     // one device buffer: cross, then d_lens (from the context's batch pool)
    size_t buf_bytes = 0;
    std::vector<uint32_t> src;  // source ids [b][s] (a shortlist decode scores them, graph.rs:98-105)
    mgb_ctx *owner = nullptr;
};

// Device buffers of freed batches, kept for the next encode: cudaFree of a few
// hundred MB takes tens of milliseconds and waits for the device, so a stream
// of batches (encode, decode, free, ...) reuses them instead. At most
// kBatchPoolBytes are kept; mgb_clear_cache and mgb_close release them.
struct PoolBuf {
    void *p;
    size_t bytes;
};
static constexpr size_t kBatchPoolBytes = 4ull << 30;

static constexpr int kLmParts = 148 * 8;  // most CTAs of a fused LM-head argmax launch (partials per row)
// Matmuls of at most this many activation rows run the reference's MMVQ
// arithmetic (candle-core's QMatMul picks MMVQ up to 8 rows, MMQ above).
static constexpr int kSmallRows = 8;
static constexpr size_t kGraphBytes = 32u << 20;

struct mgb_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    mgb_options opts{};
    Config cfg;
    uint8_t *arena = nullptr;
    size_t arena_bytes = 0;
    Matrix embed;
    std::vector<EncLayer> enc;
    std::vector<DecLayer> dec;
    Norm enc_norm, dec_norm;
    float *pos = nullptr;
    float embed_scale = 1.0f;
    uint64_t launches = 0;
    int alloc_count = 0;
    bool inject_armed = false;  // fault injection counts allocations made after mgb_open
    bool capture = true;
    uint64_t clock = 0;
    std::vector<std::unique_ptr<StaticState>> cache;
    std::vector<PoolBuf> batch_pool;  // freed batches' buffers
    size_t batch_pool_bytes = 0;
    std::unordered_set<mgb_batch *> batches;  // live batches (detached by mgb_close)
    // vocabulary shortlists (GGUF nllb.shortlist.<code> + lm_head.<code>.weight,
    // convert.rs:218-232; model.rs:229-250): sorted ids and the reduced LM head
    struct Shortlist {
        std::string code;
        std::vector<uint32_t> ids;
        Matrix W;
        const uint32_t *d_ids = nullptr;
    };
    std::vector<Shortlist> shortlists;
    size_t weight_bytes = 0, step_bytes = 0;
    uint32_t *d_err = nullptr;  // device-side error flags (a bounded wait ran out)
    // Narrowest token tile of the tensor-core matmul; 0 (the default) chooses by
    // the number of open contexts on the device (tc_floor); MGB_TC_MIN_NT sets it.
    int tc_min_nt = 0;
    // Matmuls with too few tiles for the SMs split their K stages (MGB_TC_SPLIT overrides).
    int tc_split = 1;
    int tc_split_stages = 4;  // fewest stages per split (MGB_TC_SPLIT_STAGES)
    int tc_split_max = 2;     // most splits of a tile (MGB_TC_SPLIT_MAX; 2 measured fastest at batch 64)
    // The decoder layers of greedy steps of at most 8 rows run as one persistent
    // kernel (1) or as one launch per operation (0, the default: measured faster
    // on B200); MGB_STEP_KERNEL overrides.
    int step_kernel = 0;
    // MGB_STEP_TRACE=<file>: the persistent kernel times its phases; each state
    // appends its per-launch averages to the file when it is freed.
    std::string step_trace;
    // Failure-path test hooks of the small-batch kernel (MGB_TEST_WAIT_NS,
    // MGB_TEST_WITHHOLD_CHUNK): a shorter limit for its bounded waits, and one
    // weight chunk of its first CTA that is never copied, so that a wait runs
    // out and the error word reports it. Off unless the variables are set.
    uint64_t test_wait_ns = kWaitNs;
    int test_withhold_chunk = -1;
    int test_withhold_topk = -1;  // ring position whose copy row 0 of the top-k kernel withholds (MGB_TEST_WITHHOLD_TOPK)
    int test_withhold_step = -1;  // the same for the persistent step kernel (MGB_TEST_WITHHOLD_STEP)
    // tensor-core FFN: the up epilogue writes the down matmul's q8_1 activations (1)
    // or f32 rows that a prep kernel quantizes (0, the default: the per-token
    // quantization in the epilogue measured slower on B200); MGB_FFN_Q8 overrides
    int ffn_q8 = 0;
    // small-batch matmuls: CTAs per cluster sharing the q8_1 quantization of the
    // input rows (1: each CTA quantizes all of them; 8 measured fastest on B200 at
    // batch 1: 0.80 vs 0.88 ms per step); MGB_SMALL_CLUSTER overrides
    int small_cluster = 8;
    int sms = 148;  // multiprocessor count of the device (one tensor-core CTA each)
    void *enc_ws = nullptr;  // encoder temporaries (grown on demand)
    size_t enc_ws_bytes = 0;
    size_t smem_optin = 227 * 1024 - 4096;  // dynamic shared memory a tensor-core CTA may take

    mgb_status dalloc(void **p, size_t bytes) {
        if (inject_armed && opts.fail_alloc_after >= 0 && alloc_count++ == opts.fail_alloc_after)
            return set_err(MGB_ERR_OOM, "injected allocation failure: CUDA_ERROR_OUT_OF_MEMORY");
        cudaError_t e = cudaMalloc(p, bytes < 256 ? 256 : bytes);
        if (e != cudaSuccess) {
            cudaGetLastError();
            *p = nullptr;
            return cuda_err(e, "cudaMalloc");
        }
        return MGB_OK;
    }
};

namespace {

template <typename F>
mgb_status launch_check(mgb_ctx *c, F &&f) {
    f();
    ++c->launches;
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_err(e, "kernel launch");
    return MGB_OK;
}

// Loads one tensor into the arena in the engine layout. `cursor` advances.
struct Loader {
    mgb_ctx *c;
    GgufFile *f;
    std::vector<uint8_t> host;  // staging image of the whole arena
    size_t cursor = 0;

    size_t reserve(size_t n) {
        cursor = (cursor + 255) / 256 * 256;
        size_t at = cursor;
        cursor += n;
        return at;
    }

    const GgufTensor *get(const std::string &name) {
        auto it = f->tensors.find(name);
        return it == f->tensors.end() ? nullptr : &it->second;
    }
};

// Two passes over the model: pass 0 sizes the arena, pass 1 fills the staging image.
struct Planner {
    Loader &L;
    int pass;
    std::vector<std::pair<const uint8_t **, size_t>> fix;  // device pointer slots -> arena offsets

    void ptr(const uint8_t **slot, size_t off) { fix.emplace_back(slot, off); }

    mgb_status dense(const std::string &name, long n, const float **out) {
        const GgufTensor *t = L.get(name);
        if (!t) return set_err(MGB_ERR_IO, "missing tensor %s", name.c_str());
        if (t->type != T_F32 || t->cols() * t->rows() != n)
            return set_err(MGB_ERR_UNSUPPORTED, "tensor %s must be f32 with %ld values", name.c_str(), n);
        size_t off = L.reserve(4 * n);
        if (pass == 1) memcpy(L.host.data() + off, t->data, 4 * n);
        ptr(reinterpret_cast<const uint8_t **>(out), off);
        return MGB_OK;
    }

    mgb_status norm(const std::string &name, long d, Norm &n) {
        TRY(dense(name + ".weight", d, &n.g));
        return dense(name + ".bias", d, &n.b);
    }

    mgb_status matrix(const std::string &name, Matrix &M, long want_rows, long want_cols, bool bias) {
        const GgufTensor *t = L.get(name + ".weight");
        if (!t) return set_err(MGB_ERR_IO, "missing tensor %s.weight", name.c_str());
        const long N = t->rows(), K = t->cols();
        if (N != want_rows || K != want_cols)
            return set_err(MGB_ERR_INVALID, "tensor %s.weight is [%ld, %ld], expected [%ld, %ld]", name.c_str(), N, K,
                           want_rows, want_cols);
        if (t->type != T_F32 && t->type != T_Q8_0 && t->type != T_Q4_K && t->type != T_Q6_K)
            return set_err(MGB_ERR_UNSUPPORTED, "tensor %s.weight: GGML type %d is not supported", name.c_str(), t->type);
        if (K % 32) return set_err(MGB_ERR_UNSUPPORTED, "tensor %s.weight: row length %ld", name.c_str(), K);
        M.type = t->type;
        M.N = (int)N;
        M.Np = (int)((N + 127) / 128 * 128);  // whole 128-row tensor-core tiles
        M.K = (int)K;
        M.nb = (int)(K / 32);
        M.nsb = (int)(K / 256);
        const int nb = M.nb, nsb = M.nsb;
        const long Np = M.Np;
        const long rb = row_bytes(t->type, K);
        M.bytes = (size_t)rb * N;
        auto slot = [&](long r, int j) { return ((size_t)(r / 32) * nb + j) * 32 + (size_t)(r % 32); };
        auto sslot = [&](long r, int sb) { return ((size_t)(r / 32) * nsb + sb) * 32 + (size_t)(r % 32); };
        // row layout (engine.h): the GGUF bytes row by row, split into aligned regions
        if (t->type == T_F32) {
            size_t off = L.reserve((size_t)4 * Np * K);
            if (pass == 1) memcpy(L.host.data() + off, t->data, (size_t)rb * N);
            ptr(&M.ra, off);
        } else if (t->type == T_Q4_K) {
            size_t off = L.reserve((size_t)Np * rb);
            if (pass == 1) memcpy(L.host.data() + off, t->data, (size_t)rb * N);
            ptr(&M.ra, off);
        } else if (t->type == T_Q8_0) {
            size_t oq = L.reserve((size_t)Np * nb * 32), od = L.reserve((size_t)Np * nb * 2);
            if (pass == 1) {
                uint8_t *hq = L.host.data() + oq, *hd = L.host.data() + od;
#pragma omp parallel for schedule(static)
                for (long r = 0; r < N; ++r)
                    for (int j = 0; j < nb; ++j) {
                        const uint8_t *blk = t->data + (size_t)r * rb + 34 * j;
                        memcpy(hd + ((size_t)r * nb + j) * 2, blk, 2);
                        memcpy(hq + ((size_t)r * nb + j) * 32, blk + 2, 32);
                    }
            }
            ptr(&M.ra, oq);
            ptr(&M.rb, od);
        } else {  // Q6_K
            size_t ol = L.reserve((size_t)Np * nsb * 128), oh = L.reserve((size_t)Np * nsb * 64);
            size_t os = L.reserve((size_t)Np * nsb * 16), od = L.reserve((size_t)Np * nsb * 2);
            if (pass == 1) {
                uint8_t *hl = L.host.data() + ol, *hh = L.host.data() + oh, *hs = L.host.data() + os,
                        *hd = L.host.data() + od;
#pragma omp parallel for schedule(static)
                for (long r = 0; r < N; ++r)
                    for (int sb = 0; sb < nsb; ++sb) {
                        const uint8_t *blk = t->data + (size_t)r * rb + 210 * sb;
                        const size_t u = (size_t)r * nsb + sb;
                        memcpy(hl + u * 128, blk, 128);
                        memcpy(hh + u * 64, blk + 128, 64);
                        memcpy(hs + u * 16, blk + 192, 16);
                        memcpy(hd + u * 2, blk + 208, 2);
                    }
            }
            ptr(&M.ra, ol);
            ptr(&M.rb, oh);
            ptr(&M.rc, os);
            ptr(&M.re, od);
        }
        // tensor-core layout
        if (t->type == T_F32) {
            // (small-batch kernels only)
        } else if (t->type == T_Q8_0) {
            size_t oq = L.reserve((size_t)Np * nb * 32), od = L.reserve((size_t)Np * nb * 2);
            if (pass == 1) {
                uint8_t *hq = L.host.data() + oq, *hd = L.host.data() + od;
#pragma omp parallel for schedule(static)
                for (long r = 0; r < N; ++r) {
                    const uint8_t *row = t->data + (size_t)r * rb;
                    for (int j = 0; j < nb; ++j) {
                        memcpy(hd + slot(r, j) * 2, row + 34 * j, 2);
                        memcpy(hq + slot(r, j) * 32, row + 34 * j + 2, 32);
                    }
                }
            }
            ptr(&M.a, oq);
            ptr(&M.b, od);
        } else if (t->type == T_Q4_K) {
            size_t oq = L.reserve((size_t)Np * nb * 16), oh = L.reserve((size_t)Np * nsb * 16);
            if (pass == 1) {
                uint8_t *hq = L.host.data() + oq, *hh = L.host.data() + oh;
#pragma omp parallel for schedule(static)
                for (long r = 0; r < N; ++r) {
                    const uint8_t *row = t->data + (size_t)r * rb;
                    uint8_t q[32];
                    for (int j = 0; j < nb; ++j) {
                        q4k_block_values(row, j, q);
                        uint8_t *dst = hq + slot(r, j) * 16;
                        for (int k = 0; k < 16; ++k) dst[k] = (uint8_t)(q[k] | (q[k + 16] << 4));
                    }
                    for (int sb = 0; sb < nsb; ++sb) memcpy(hh + sslot(r, sb) * 16, row + 144 * sb, 16);
                }
            }
            ptr(&M.a, oq);
            ptr(&M.b, oh);
        } else {  // Q6_K
            size_t ol = L.reserve((size_t)Np * nb * 16), oh = L.reserve((size_t)Np * nb * 8);
            size_t os = L.reserve((size_t)Np * nb * 2), od = L.reserve((size_t)Np * nsb * 2);
            if (pass == 1) {
                uint8_t *hl = L.host.data() + ol, *hh = L.host.data() + oh, *hs = L.host.data() + os,
                        *hd = L.host.data() + od;
#pragma omp parallel for schedule(static)
                for (long r = 0; r < N; ++r) {
                    const uint8_t *row = t->data + (size_t)r * rb;
                    uint8_t q[32];
                    for (int j = 0; j < nb; ++j) {
                        q6k_block_values(row, j, q);
                        const size_t bi = slot(r, j);
                        for (int k = 0; k < 16; ++k) hl[bi * 16 + k] = (uint8_t)((q[k] & 0xf) | ((q[k + 16] & 0xf) << 4));
                        uint32_t A = 0, B = 0;
                        for (int k = 0; k < 16; ++k) {
                            const int i = k / 4, bb = k % 4;
                            A |= (uint32_t)(q[k] >> 4) << (8 * bb + 2 * i);
                            B |= (uint32_t)(q[k + 16] >> 4) << (8 * bb + 2 * i);
                        }
                        memcpy(hh + bi * 8, &A, 4);
                        memcpy(hh + bi * 8 + 4, &B, 4);
                        const uint8_t *sc = row + (j / 8) * 210 + 192;
                        hs[bi * 2] = sc[2 * (j % 8)];
                        hs[bi * 2 + 1] = sc[2 * (j % 8) + 1];
                    }
                    for (int sb = 0; sb < nsb; ++sb) memcpy(hd + sslot(r, sb) * 2, row + 210 * sb + 208, 2);
                }
            }
            ptr(&M.a, ol);
            ptr(&M.b, oh);
            ptr(&M.c, os);
            ptr(&M.e, od);
        }
        if (bias) TRY(dense(name + ".bias", N, &M.bias));
        return MGB_OK;
    }
};

uint32_t next_pow2(uint32_t n) {
    uint32_t p = 1;
    while (p < n) p <<= 1;
    return p;
}

}  // namespace

// bucket(n, min, max) = max(min(next_pow2(max(n, min)), max), n) (graph.rs:138-140)
static int bucket(int n, int mn, int mx) {
    int v = (int)next_pow2((uint32_t)std::max(n, mn));
    return std::max(std::min(v, mx), n);
}

static mgb_status load_model(mgb_ctx *c, const char *path) {
    GgufFile f;
    TRY(parse_gguf(path, f));
    auto u = [&](const char *k, int &dst, bool required = true) -> mgb_status {
        auto it = f.u32.find(k);
        if (it == f.u32.end()) {
            if (required) return set_err(MGB_ERR_IO, "missing GGUF metadata key '%s'", k);
            return MGB_OK;
        }
        dst = (int)it->second;
        return MGB_OK;
    };
    Config &g = c->cfg;
    TRY(u("nllb.vocab_size", g.V));
    TRY(u("nllb.embedding_length", g.d));
    TRY(u("nllb.encoder.block_count", g.enc_layers));
    TRY(u("nllb.decoder.block_count", g.dec_layers));
    TRY(u("nllb.encoder.attention.head_count", g.enc_heads));
    TRY(u("nllb.decoder.attention.head_count", g.dec_heads));
    TRY(u("nllb.encoder.feed_forward_length", g.enc_ffn));
    TRY(u("nllb.decoder.feed_forward_length", g.dec_ffn));
    TRY(u("nllb.context_length", g.max_pos));
    TRY(u("nllb.scale_embedding", g.scale_embedding));
    TRY(u("nllb.max_length", g.max_length));
    TRY(u("tokenizer.ggml.padding_token_id", g.pad));
    TRY(u("tokenizer.ggml.eos_token_id", g.eos));
    TRY(u("tokenizer.ggml.decoder_start_token_id", g.start));
    TRY(u("tokenizer.ggml.bos_token_id", g.bos, false));
    // d_model <= 2048 as the reference's fused kernels (kernels.rs:44-47, 89-91)
    if (g.d % 32 || g.d % g.dec_heads || g.d % g.enc_heads || g.d > 2048)
        return set_err(MGB_ERR_UNSUPPORTED, "d_model %d with %d/%d heads", g.d, g.enc_heads, g.dec_heads);

    Loader L{c, &f};
    const int d = g.d;
    c->shortlists.clear();
    for (const auto &kv : f.u32arr) {
        const std::string pre = "nllb.shortlist.";
        if (kv.first.compare(0, pre.size(), pre) != 0) continue;
        mgb_ctx::Shortlist sl;
        sl.code = kv.first.substr(pre.size());
        sl.ids = kv.second;
        for (size_t i = 0; i < sl.ids.size(); ++i)
            if (sl.ids[i] >= (uint32_t)g.V || (i && sl.ids[i] <= sl.ids[i - 1]))
                return set_err(MGB_ERR_IO, "shortlist %s: ids not sorted within the vocabulary", sl.code.c_str());
        if (sl.ids.empty()) continue;
        c->shortlists.push_back(std::move(sl));
    }
    c->enc.resize(g.enc_layers);
    c->dec.resize(g.dec_layers);
    for (int pass = 0; pass < 2; ++pass) {
        if (pass == 1) L.host.assign(L.cursor + 256, 0);
        L.cursor = 0;
        Planner P{L, pass};
        TRY(P.matrix("token_embd", c->embed, g.V, d, false));
        char nm[128];
        for (int i = 0; i < g.enc_layers; ++i) {
            EncLayer &l = c->enc[i];
            auto n = [&](const char *s) { snprintf(nm, sizeof nm, "enc.blk.%d.%s", i, s); return std::string(nm); };
            TRY(P.norm(n("attn_norm"), d, l.attn_norm));
            TRY(P.norm(n("ffn_norm"), d, l.ffn_norm));
            TRY(P.matrix(n("attn_qkv"), l.qkv, 3 * d, d, true));
            TRY(P.matrix(n("attn_out"), l.out, d, d, true));
            TRY(P.matrix(n("ffn_up"), l.up, g.enc_ffn, d, true));
            TRY(P.matrix(n("ffn_down"), l.down, d, g.enc_ffn, true));
        }
        for (int i = 0; i < g.dec_layers; ++i) {
            DecLayer &l = c->dec[i];
            auto n = [&](const char *s) { snprintf(nm, sizeof nm, "dec.blk.%d.%s", i, s); return std::string(nm); };
            TRY(P.norm(n("attn_norm"), d, l.attn_norm));
            TRY(P.norm(n("cross_attn_norm"), d, l.cross_norm));
            TRY(P.norm(n("ffn_norm"), d, l.ffn_norm));
            TRY(P.matrix(n("attn_qkv"), l.qkv, 3 * d, d, true));
            TRY(P.matrix(n("attn_out"), l.out, d, d, true));
            TRY(P.matrix(n("cross_attn_q"), l.cq, d, d, true));
            TRY(P.matrix(n("cross_attn_kv"), l.ckv, 2 * d, d, true));
            TRY(P.matrix(n("cross_attn_out"), l.co, d, d, true));
            TRY(P.matrix(n("ffn_up"), l.up, g.dec_ffn, d, true));
            TRY(P.matrix(n("ffn_down"), l.down, d, g.dec_ffn, true));
        }
        TRY(P.norm("enc.output_norm", d, c->enc_norm));
        TRY(P.norm("dec.output_norm", d, c->dec_norm));
        for (mgb_ctx::Shortlist &sl : c->shortlists) {
            TRY(P.matrix("lm_head." + sl.code, sl.W, (long)sl.ids.size(), d, false));
            const size_t o = L.reserve(4 * sl.ids.size());
            if (pass == 1) memcpy(L.host.data() + o, sl.ids.data(), 4 * sl.ids.size());
            P.ptr(reinterpret_cast<const uint8_t **>(const_cast<const uint32_t **>(&sl.d_ids)), o);
        }
        // Sinusoidal position table [max_pos + pad + 1, d] (model.rs:325-340, 361-366).
        const int n_pos = g.max_pos + g.pad + 1;
        size_t off = L.reserve((size_t)n_pos * d * 4);
        if (pass == 1) {
            float *tab = reinterpret_cast<float *>(L.host.data() + off);
            const int half = d / 2;
            const double st = std::log(10000.0) / ((double)half - 1.0);
            for (int p = 0; p < n_pos; ++p)
                for (int i = 0; i < half; ++i) {
                    if (p == g.pad) continue;
                    const double a = (double)p * std::exp(-(double)i * st);
                    tab[(size_t)p * d + i] = (float)std::sin(a);
                    tab[(size_t)p * d + half + i] = (float)std::cos(a);
                }
        }
        P.ptr(reinterpret_cast<const uint8_t **>(const_cast<const float **>(&c->pos)), off);
        if (pass == 1) {
            void *arena = nullptr;
            TRY(c->dalloc(&arena, L.cursor));
            c->arena = (uint8_t *)arena;
            c->arena_bytes = L.cursor;
            CK(cudaMemcpy(c->arena, L.host.data(), L.cursor, cudaMemcpyHostToDevice));
            for (auto &fx : P.fix) *fx.first = c->arena + fx.second;
        }
    }
    c->embed_scale = g.scale_embedding ? (float)std::sqrt((double)d) : 1.0f;
    c->weight_bytes = c->arena_bytes;
    size_t step = c->embed.bytes;
    for (auto &l : c->dec) step += l.qkv.bytes + l.out.bytes + l.cq.bytes + l.co.bytes + l.up.bytes + l.down.bytes;
    c->step_bytes = step;
    return MGB_OK;
}

// ---------------------------------------------------------------------------
// Kernel launchers

// Launch with programmatic stream serialization: the kernel may begin (and
// prefetch) while its predecessor finishes; it waits in griddepcontrol.wait.
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k, args...);
}

// launch_pdl with thread-block clusters of `cluster` CTAs along x (grid.x a multiple of it).
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl_cluster(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                      int cluster, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = (unsigned)cluster;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = cluster > 1 ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, k, args...);
}

// Raises a kernel's dynamic shared-memory limit to the full 227 KB once
// (before any graph capture: the first step of every shape runs eagerly).
// (per device: one process may drive several GPUs, one context each)
template <typename... KArgs>
static cudaError_t allow_smem(void (*k)(KArgs...), size_t bytes) {
    static std::mutex mu;
    static std::set<std::pair<int, const void *>> done;
    if (bytes <= 48 * 1024) return cudaSuccess;
    int dev = 0, optin = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    if (done.count({dev, (const void *)k})) return cudaSuccess;
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaFuncAttributes fa{};
    cudaError_t e = cudaFuncGetAttributes(&fa, k);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - (int)fa.sharedSizeBytes);
    if (e == cudaSuccess) done.insert({dev, (const void *)k});
    return e;
}

template <typename KV>
static mgb_status attend(mgb_ctx *c, AttnArgs a) {
    const long tasks = (long)a.rows * a.H * a.queries;
    const int grid = (int)((tasks + 3) / 4);
    // 4 warps: score/probability rows (max_keys floats) + a 64-key V staging tile
    const size_t sh = (size_t)4 * a.max_keys * sizeof(float) + (size_t)4 * 64 * a.hd * sizeof(KV);
    auto go = [&](auto kern) -> mgb_status {
        cudaError_t e = allow_smem(kern, sh);
        if (e == cudaSuccess) e = launch_pdl(kern, dim3(grid), dim3(128), sh, c->stream, a);
        ++c->launches;
        if (e != cudaSuccess) return cuda_err(e, "attention launch");
        return MGB_OK;
    };
    // single-query attention of a small decode batch releases the next kernel late
    const bool late = a.queries == 1 && a.rows <= kSmallRows;
    switch (a.hd) {
        case 16: return late ? go(attend_kernel<KV, 16, true>) : go(attend_kernel<KV, 16, false>);
        case 32: return late ? go(attend_kernel<KV, 32, true>) : go(attend_kernel<KV, 32, false>);
        case 64: return late ? go(attend_kernel<KV, 64, true>) : go(attend_kernel<KV, 64, false>);
        case 128: return late ? go(attend_kernel<KV, 128, true>) : go(attend_kernel<KV, 128, false>);
    }
    return set_err(MGB_ERR_UNSUPPORTED, "head dimension %d", a.hd);
}

// Small-batch matmul (smallmm.cuh). NC = the launch's rows rounded up to a
// power of two; the MMVQ warp count follows from it as in candle's launch
// table (4 warps for 1-4 rows, 2 for 5-8). At least 8 weight rows per CTA, at
// most two CTAs per SM; stages of 32 rows (R = 4 rows per warp) while that
// stays within 32 KB, else 8 rows.
template <int TYPE, int EPI, int MODE, int NC, int R>
static cudaError_t small_launch(mgb_ctx *c, const SmallArgs &a, int grid, size_t smem) {
    auto kern = small_mm_kernel<TYPE, EPI, MODE, NC, NC <= 4 ? 4 : 2, R>;
    cudaError_t e = allow_smem(kern, smem);
    return e == cudaSuccess ? launch_pdl_cluster(kern, dim3(grid), dim3(256), smem, c->stream, a.cluster, a) : e;
}

template <int TYPE, int EPI, int MODE, int NC>
static cudaError_t small_launch_r(mgb_ctx *c, const SmallArgs &a, int grid, size_t smem, int R) {
    return R == 4 ? small_launch<TYPE, EPI, MODE, NC, 4>(c, a, grid, smem)
                  : small_launch<TYPE, EPI, MODE, NC, 1>(c, a, grid, smem);
}

template <int TYPE, int EPI, int MODE>
static mgb_status small_t(mgb_ctx *c, const GemvArgs &g, const PrepArgs &p, int *ctas, int cls) {
    const Matrix &W = g.W;
    const int RB = row_bytes_of(TYPE, W.K), groups = W.Np / 8;
    const int R = TYPE != T_F32 && 32 * RB <= 32 * 1024 ? 4 : 1;
    int grid = std::min(groups, 2 * c->sms);
    const int rpc = (groups + grid - 1) / grid * 8;
    grid = (W.Np + rpc - 1) / rpc;
    // clusters share the activation quantization (CTAs past the rows only quantize);
    // not the LM head, a long weight stream that runs slower in clusters (co-scheduling)
    const int cluster = TYPE != T_F32 && EPI != EPI_ARGMAX && c->small_cluster > 1 ? c->small_cluster : 1;
    grid = (grid + cluster - 1) / cluster * cluster;
    if (ctas) *ctas = grid;
    // launches of at most 8 activation rows (more only for F32 weights)
    for (int n0 = 0; n0 < g.rows; n0 += kSmallRows) {
        const int here = std::min(kSmallRows, g.rows - n0);
        // (5-8 rows of the reference's call: 2 warps, the 8-column variant)
        const int NC = cls > 4 ? 8 : here <= 1 ? 1 : here <= 2 ? 2 : here <= 4 ? 4 : 8;
        SmallArgs a{};
        a.g = g;
        a.p = p;
        a.n0 = n0;
        a.rows_per_cta = rpc;
        const int nch = (rpc + 8 * R - 1) / (8 * R);
        a.stages = TYPE == T_F32 ? 0 : std::min(3, nch);
        a.err = c->d_err;
        a.wait_ns = c->test_wait_ns;
        a.withhold_chunk = c->test_withhold_chunk;
        a.cluster = cluster;
        const size_t act = small_act_bytes(NC, W.K, TYPE, MODE), sb = (size_t)8 * R * RB;
        while (a.stages > 1 && (size_t)a.stages * sb + act > c->smem_optin) --a.stages;
        const size_t smem = (size_t)a.stages * sb + act;
        if (smem > c->smem_optin)
            return set_err(MGB_ERR_UNSUPPORTED, "small-batch matmul of a %d-value row needs %zu B of shared memory",
                           W.K, smem);
        cudaError_t e;
        switch (NC) {
            case 1: e = small_launch_r<TYPE, EPI, MODE, 1>(c, a, grid, smem, R); break;
            case 2: e = small_launch_r<TYPE, EPI, MODE, 2>(c, a, grid, smem, R); break;
            case 4: e = small_launch_r<TYPE, EPI, MODE, 4>(c, a, grid, smem, R); break;
            default: e = small_launch_r<TYPE, EPI, MODE, 8>(c, a, grid, smem, R); break;
        }
        ++c->launches;
        if (e != cudaSuccess) return cuda_err(e, "small-batch matmul launch");
    }
    return MGB_OK;
}

// y = W . act(p) with the reference's MMVQ arithmetic (at most 8 rows; F32
// weights any number). cls: the rows of the reference's call (the MMVQ warp
// count; 0 = g.rows). *ctas: CTAs of the launch (argmax partials per row).
template <int EPI, int MODE>
static mgb_status small_mm(mgb_ctx *c, GemvArgs g, PrepArgs p, int *ctas = nullptr, int cls = 0) {
    p.rows = g.rows;
    p.K = g.W.K;
    if (!cls) cls = g.rows;
    switch (g.W.type) {
        case T_F32: return small_t<T_F32, EPI, MODE>(c, g, p, ctas, cls);
        case T_Q8_0: return small_t<T_Q8_0, EPI, MODE>(c, g, p, ctas, cls);
        case T_Q4_K: return small_t<T_Q4_K, EPI, MODE>(c, g, p, ctas, cls);
        case T_Q6_K: return small_t<T_Q6_K, EPI, MODE>(c, g, p, ctas, cls);
    }
    return set_err(MGB_ERR_UNSUPPORTED, "matrix type %d", g.W.type);
}

static bool tc_ok(const Matrix &W) { return W.type == T_Q8_0 || W.type == T_Q4_K || W.type == T_Q6_K; }

// Tensor-core path: q8_1 activations of `rows` rows into `act` (one CTA per row).
template <int MODE>
static mgb_status qprep_row(mgb_ctx *c, PrepArgs p, const QAct &act) {
    auto kern = qprep_row_kernel<MODE>;
    const size_t sh = (size_t)p.K * 4 + (MODE != PREP_PLAIN ? (size_t)p.K * 8 : 0);  // row; gamma, beta
    cudaError_t e = allow_smem(kern, sh);
    // a warp per 32-value block (up to 1024 threads): the blocks' q8_1 reductions run side by side
    const int threads = std::min(1024, std::max(256, p.K));
    if (e == cudaSuccess) e = launch_pdl(kern, dim3(p.rows), dim3(threads), sh, c->stream, p, act);
    ++c->launches;
    return e == cudaSuccess ? MGB_OK : cuda_err(e, "activation prep launch");
}

template <int TYPE>
static size_t tc_smem_t(int nt) {
    switch (nt) {
        case 8: return gemm_tc_smem<TYPE, 8>();
        case 16: return gemm_tc_smem<TYPE, 16>();
        case 32: return gemm_tc_smem<TYPE, 32>();
        default: return gemm_tc_smem<TYPE, 64>();
    }
}

static size_t tc_smem(int type, int nt) {
    switch (type) {
        case T_Q8_0: return tc_smem_t<T_Q8_0>(nt);
        case T_Q4_K: return tc_smem_t<T_Q4_K>(nt);
        default: return tc_smem_t<T_Q6_K>(nt);
    }
}

// Open contexts per device. Every tensor-core CTA holds an SM, and narrow token
// tiles repeat a weight tile's conversion once per tile: the fastest launch
// alone on a GPU, but the most SM time per token. With one context the matmuls
// choose the fastest launch; the more contexts decode concurrently
// (dp.StreamPool), the more the GPU's SM time is the bound and the wider the
// narrowest tile: 16 tokens for 2-3 contexts, 32 from 4 (or one tile for a
// smaller batch). Batch-64 decode on NLLB-600M q4_k_m, B200, tokens/s by floor
// 8 / 16 / 32: 2 contexts 56.5k / 60.2k / 53.0k, 4 contexts 64.1k / 69.1k /
// 70.7k; 8 contexts with 32: 83.9k; one context loses 30 % with 32. The floor
// is read when a step is launched or captured: a CUDA graph keeps the tiles of
// its capture (dp.StreamPool opens all its contexts before the first decode).
static std::mutex g_ctx_mu;
static std::map<int, int> g_ctx_open;

static int contexts_on(int device) {
    std::lock_guard<std::mutex> lock(g_ctx_mu);
    auto it = g_ctx_open.find(device);
    return it == g_ctx_open.end() ? 0 : it->second;
}

static void count_context(int device, int delta) {
    std::lock_guard<std::mutex> lock(g_ctx_mu);
    g_ctx_open[device] += delta;
}

static int tc_floor(const mgb_ctx *c, int rows) {
    if (c->tc_min_nt > 0) return c->tc_min_nt;
    const int open = contexts_on(c->device);
    if (open <= 1) return 8;
    const int cap = open >= 4 ? 32 : 16;
    int f = 8;
    while (f < cap && f < rows) f *= 2;
    return f;
}

// Token tile (activation rows per tile, at least min_nt) of a tensor-core
// matmul: the one that needs the fewest waves of tiles over the SMs, on a tie
// the narrowest, whose tiles finish soonest; persistent CTAs, one per SM.
static void tc_shape(const Matrix &W, int rows, int sms, int min_nt, int &nt, int &grid) {
    const int row_tiles = W.Np / 128;
    long best = 0;
    nt = 0;
    for (int cand : {8, 16, 32, 64}) {
        if (cand < min_nt && cand != 64) continue;
        const long waves = ((long)row_tiles * ((rows + cand - 1) / cand) + sms - 1) / sms;
        if (!nt || waves < best) {
            nt = cand;
            best = waves;
        }
    }
    grid = (int)std::min<long>((long)row_tiles * ((rows + nt - 1) / nt), sms);
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
    });
    return fn;
}

// A tensor map of 8-byte words: dims[0] innermost; strides in bytes for dims 1..
static mgb_status tmap(CUtensorMap *m, const void *base, int rank, const uint64_t *dims, const uint64_t *strides,
                       const uint32_t *box, bool weights) {
    EncodeTiledFn fn = encode_tiled();
    if (!fn) return set_err(MGB_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
    cuuint64_t gd[4], gs[3];
    cuuint32_t bx[4], es[4];
    for (int i = 0; i < rank; ++i) {
        gd[i] = dims[i];
        bx[i] = box[i];
        es[i] = 1;
        if (i) gs[i - 1] = strides[i - 1];
    }
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, (cuuint32_t)rank, const_cast<void *>(base), gd, gs, bx, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                    weights ? CU_TENSOR_MAP_L2_PROMOTION_L2_256B : CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_err(MGB_ERR_CUDA, "tensor map encoding failed (%d)", (int)r);
    return MGB_OK;
}

// The launch's tensor maps (layouts: engine.h Matrix and QAct, gemm_tc.cuh tc::Maps).
static mgb_status make_maps(const Matrix &W, const QAct &x, int nt, tc::Maps &m) {
    memset(&m, 0, sizeof m);
    const uint64_t G = (uint64_t)W.Np / 32, nb = W.nb, nsb = W.nsb;
    // one weight region: X words per (group, block-or-super-block) slice, n slices, boxes of k slices
    auto region = [&](CUtensorMap *mp, const uint8_t *base, uint64_t X, uint64_t n, uint32_t k) -> mgb_status {
        const uint64_t dims[3] = {X, n, G}, str[2] = {X * 8, X * 8 * n};
        const uint32_t box[3] = {(uint32_t)X, k, 4};
        return tmap(mp, base, 3, dims, str, box, true);
    };
    switch (W.type) {
        case T_Q8_0:
            TRY(region(&m.w[0], W.a, 128, nb, 8));
            TRY(region(&m.w[1], W.b, 8, nb, 8));
            break;
        case T_Q4_K:
            TRY(region(&m.w[0], W.a, 64, nb, 8));
            TRY(region(&m.w[1], W.b, 64, nsb, 1));
            break;
        case T_Q6_K:
            TRY(region(&m.w[0], W.a, 64, nb, 8));
            TRY(region(&m.w[1], W.b, 32, nb, 8));
            TRY(region(&m.w[2], W.c, 8, nb, 8));
            TRY(region(&m.w[3], W.e, 8, nsb, 1));
            break;
        default:
            return set_err(MGB_ERR_UNSUPPORTED, "tensor-core matmul of type %d", W.type);
    }
    const uint64_t rs = (uint64_t)x.rs;
    {
        const uint64_t dims[3] = {32, rs / 8, nb}, str[2] = {256, rs * 32};
        const uint32_t box[3] = {32, (uint32_t)nt / 8, 8};
        TRY(tmap(&m.xq, x.tq, 3, dims, str, box, false));
    }
    {
        // records: one float2 (8-byte word) per (block, row)
        const uint64_t dims[2] = {rs, nb}, str[1] = {rs * 8};
        const uint32_t box[2] = {(uint32_t)nt, 8};
        TRY(tmap(&m.xr, x.trec, 2, dims, str, box, false));
    }
    return MGB_OK;
}

template <int TYPE, int EPI>
static mgb_status gemm_tc_t(mgb_ctx *c, const tc::Args &a, int nt, int grid) {
    const size_t sh = tc_smem(TYPE, nt);
    auto go = [&](auto kern) -> cudaError_t {
        cudaError_t e = allow_smem(kern, sh);
        return e == cudaSuccess ? launch_pdl(kern, dim3(grid), dim3(tc::kThreads), sh, c->stream, a) : e;
    };
    cudaError_t e;
    switch (nt) {
        case 8: e = go(gemm_tc_kernel<TYPE, EPI, 8>); break;
        case 16: e = go(gemm_tc_kernel<TYPE, EPI, 16>); break;
        case 32: e = go(gemm_tc_kernel<TYPE, EPI, 32>); break;
        default: e = go(gemm_tc_kernel<TYPE, EPI, 64>); break;
    }
    ++c->launches;
    return e == cudaSuccess ? MGB_OK : cuda_err(e, "tensor-core matmul launch");
}

// y = W . x for `rows` activation rows (q8_1 in `act`, written by qprep_row or
// the attention kernel) on the tensor cores, epilogue EPI, the reference's MMQ
// arithmetic. The LM head (ARGMAX) runs in launches of at most 64 rows (one
// token tile each); *ctas returns its CTA count, the partial count per row.
template <int EPI>
static mgb_status gemm_tc(mgb_ctx *c, const Matrix &W, const QAct &act, int rows, const GemvArgs &g,
                          int *ctas = nullptr, const SplitBufs *split = nullptr) {
    if (!tc_ok(W)) return set_err(MGB_ERR_UNSUPPORTED, "tensor-core matmul of type %d", W.type);
    const int chunk = EPI == EPI_ARGMAX ? 64 : rows;
    for (int t0 = 0; t0 < rows; t0 += chunk) {
        const int n = std::min(chunk, rows - t0);
        tc::Args a;
        memset(&a, 0, sizeof a);
        a.W = W;
        a.rows = n;
        a.tok0 = t0;
        a.g = g;
        a.g.W = W;
        a.g.rows = n;
        a.err = c->d_err;
        int nt, grid;
        const int floor_nt = tc_floor(c, n);
        tc_shape(W, n, c->sms, floor_nt, nt, grid);
        if (EPI == EPI_ARGMAX) {
            if (a.g.logits) a.g.logits += (size_t)t0 * W.N;
            a.g.part_v += (size_t)t0 * grid;
            a.g.part_i += (size_t)t0 * grid;
        }
        a.row_tiles = W.Np / 128;
        a.splits = 1;
        if (split && split->part && EPI != EPI_ARGMAX) {
            // Too few tiles for the SMs: split the stages (2 or 4 ways) where they divide, each split keeping
            // tc_split_stages or more. Token tile and split count together: the fewest stages per CTA times
            // waves over the SMs (on a tie the narrowest tile), e.g. the 16-stage FFN down at batch 64 runs as
            // 16-token tiles split 4 ways (4 stages a CTA) rather than 8-token tiles split 2 ways (8).
            const int ns = (W.nb + 7) / 8;
            const int nu = W.type == T_Q8_0 ? W.nb : W.nb / 2;
            long best = 0;
            int best_nt = nt, best_splits = 1;
            for (int cand : {8, 16, 32, 64}) {
                if (cand < floor_nt && cand != 64) continue;
                const int tt = (n + cand - 1) / cand, tiles = a.row_tiles * tt;
                int sp = 1;
                while (sp * 2 <= c->tc_split_max && tiles * sp * 2 <= c->sms && ns % (sp * 2) == 0 &&
                       ns / (sp * 2) >= c->tc_split_stages)
                    sp *= 2;
                if (sp > 1 && (size_t)tt * cand * W.Np * nu > split->part_units) sp = 1;
                const long waves = ((long)tiles * sp + c->sms - 1) / c->sms;
                const long cost = waves * (ns / sp);
                if (best == 0 || cost < best) {
                    best = cost;
                    best_nt = cand;
                    best_splits = sp;
                }
            }
            nt = best_nt;
            a.splits = best_splits;
            const int tiles = a.row_tiles * ((n + nt - 1) / nt);
            grid = (int)std::min<long>((long)tiles * a.splits, c->sms);
            if (a.splits > 1) {
                a.kpart = split->part;
                a.kcount = split->count;
            }
        }
        a.tok_tiles = (n + nt - 1) / nt;
        if (ctas) *ctas = grid;
        TRY(make_maps(W, act, nt, a.m));
        switch (W.type) {
            case T_Q8_0: TRY((gemm_tc_t<T_Q8_0, EPI>(c, a, nt, grid))); break;
            case T_Q4_K: TRY((gemm_tc_t<T_Q4_K, EPI>(c, a, nt, grid))); break;
            default: TRY((gemm_tc_t<T_Q6_K, EPI>(c, a, nt, grid))); break;
        }
    }
    return MGB_OK;
}

// q8_1 activation buffers of the tensor-core path: tiles and records for rows
// padded to 64 and rows of up to kmax values.
static mgb_status alloc_tc_act(mgb_ctx *c, int rows, int kmax, QAct &a, std::vector<void *> &allocs, size_t *bytes) {
    const int rp = (rows + 63) / 64 * 64, nbm = kmax / 32;
    auto A = [&](void **p, size_t n) -> mgb_status {
        TRY(c->dalloc(p, n));
        allocs.push_back(*p);
        if (bytes) *bytes += n;
        CK(cudaMemsetAsync(*p, 0, n, c->stream));
        return MGB_OK;
    };
    TRY(A((void **)&a.tq, (size_t)nbm * rp * 32));
    TRY(A((void **)&a.trec, (size_t)nbm * rp * 8));
    a.rs = rp;
    return MGB_OK;
}

// ---------------------------------------------------------------------------
// Static state (graph.rs:23-135)

// Appends a state's phase timing (per-launch averages, microseconds) to its file.
static void dump_trace(StaticState *st) {
    const size_t n = st->phase_host.size();
    std::vector<unsigned long long> t(8 * n + 1);
    if (cudaMemcpy(t.data(), st->trace, 8 * t.size(), cudaMemcpyDeviceToHost) != cudaSuccess || !t[8 * n]) return;
    FILE *f = fopen(st->trace_path.c_str(), "a");
    if (!f) return;
    const double L = (double)t[8 * n], ctas = st->step_ctas > 0 ? st->step_ctas : 1;
    fprintf(f, "# rows %d, launches %.0f: phase kind epi N K rsel | staged stats act chunk work barrier | cta_mean_us\n",
            st->b, L);
    for (size_t i = 0; i < n; ++i) {
        const StepPhase &p = st->phase_host[i];
        fprintf(f, "%zu %s %d %d %d %d |", i, p.kind == PH_MM ? "mm" : "attn", p.epi, p.W.N, p.W.K, p.rsel);
        for (int k = 0; k < 6; ++k) fprintf(f, " %.2f", t[8 * i + k] / L / 1e3);
        fprintf(f, " | %.2f\n", t[8 * i + 6] / L / ctas / 1e3);
    }
    fclose(f);
}

static void free_state(StaticState *st) {
    if (st->trace) dump_trace(st);
    if (st->exec) cudaGraphExecDestroy(st->exec);
    for (void *p : st->allocs) cudaFree(p);
    st->allocs.clear();
}

static mgb_status new_state(mgb_ctx *c, int b, int s, int m, StaticState **out) {
    auto st = std::make_unique<StaticState>();
    st->b = b;
    st->s = s;
    st->m = m;
    const Config &g = c->cfg;
    const int d = g.d, H = g.dec_heads, hd = d / H;
    auto A = [&](void **p, size_t n) -> mgb_status {
        TRY(c->dalloc(p, n));
        st->allocs.push_back(*p);
        st->bytes += n;
        return MGB_OK;
    };
    TRY(A((void **)&st->ids, 4 * b));
    TRY(A((void **)&st->step, 4));
    TRY(A((void **)&st->out, (size_t)4 * b * m));
    TRY(A((void **)&st->lens, 4 * b));
    TRY(A((void **)&st->finished, b));
    TRY(A((void **)&st->x, (size_t)4 * b * d));
    TRY(A((void **)&st->q, (size_t)4 * b * d));
    TRY(A((void **)&st->a, (size_t)4 * b * d));
    TRY(A((void **)&st->u, (size_t)4 * b * g.dec_ffn));
    st->kc.resize(g.dec_layers);
    st->vc.resize(g.dec_layers);
    st->ck.resize(g.dec_layers);
    st->cv.resize(g.dec_layers);
    for (int l = 0; l < g.dec_layers; ++l) {
        TRY(A((void **)&st->kc[l], (size_t)2 * b * H * m * hd));
        TRY(A((void **)&st->vc[l], (size_t)2 * b * H * m * hd));
        TRY(A((void **)&st->ck[l], (size_t)2 * b * H * s * hd));
        TRY(A((void **)&st->cv[l], (size_t)2 * b * H * s * hd));
        CK(cudaMemsetAsync(st->kc[l], 0, (size_t)2 * b * H * m * hd, c->stream));
        CK(cudaMemsetAsync(st->vc[l], 0, (size_t)2 * b * H * m * hd, c->stream));
        CK(cudaMemsetAsync(st->ck[l], 0, (size_t)2 * b * H * s * hd, c->stream));
        CK(cudaMemsetAsync(st->cv[l], 0, (size_t)2 * b * H * s * hd, c->stream));
    }
    TRY(A((void **)&st->part_v, (size_t)4 * b * kLmParts));
    TRY(A((void **)&st->part_i, (size_t)4 * b * kLmParts));
    if (tc_ok(c->dec[0].qkv)) {  // (small batches too: beam prefills can take the MMQ path)
        TRY(alloc_tc_act(c, b, std::max(d, g.dec_ffn), st->act, st->allocs, &st->bytes));
        TRY(alloc_tc_act(c, b, g.dec_ffn, st->act2, st->allocs, &st->bytes));
    }
    if (b > kSmallRows && tc_ok(c->dec[0].qkv)) {
        // split-K: the largest (rows x units) of the step's matrices, rows padded to 64
        size_t pu = 0;
        for (const DecLayer &L : c->dec)
            for (const Matrix *M : {&L.qkv, &L.out, &L.cq, &L.co, &L.up, &L.down})
                pu = std::max(pu, (size_t)M->Np * ((b + 63) / 64 * 64) * (M->type == T_Q8_0 ? M->nb : M->nb / 2));
        st->split.part_units = pu;
        TRY(A((void **)&st->split.part, 8 * pu));
        TRY(A((void **)&st->split.count, 4 * 4096));
        CK(cudaMemsetAsync(st->split.count, 0, 4 * 4096, c->stream));
    }
    *out = st.release();
    return MGB_OK;
}

static PrepArgs prep_src(const float *x, const Norm *n) {
    PrepArgs p{};
    p.x = x;
    if (n) {
        p.gamma = n->g;
        p.beta = n->b;
    }
    return p;
}

static GemvArgs mm_out(const Matrix &W, int rows) {
    GemvArgs g{};
    g.W = W;
    g.rows = rows;
    return g;
}

// A matmul of the decode step or the encoder: the reference's MMVQ arithmetic
// (small-batch kernel) when its call has at most 8 rows (cls, default the
// rows computed here) or for F32 weights, else MMQ on the tensor cores with the
// activations prepared by qprep_row into `act`.
template <int EPI, int MODE>
static mgb_status matmul(mgb_ctx *c, const GemvArgs &g, const PrepArgs &p, const QAct *act, int *ctas = nullptr,
                         const SplitBufs *split = nullptr, int cls = 0) {
    if (!cls) cls = g.rows;
    if (cls <= kSmallRows || !tc_ok(g.W)) return small_mm<EPI, MODE>(c, g, p, ctas, cls);
    if (!act || !act->tq) return set_err(MGB_ERR_INVALID, "tensor-core activation buffers missing");
    PrepArgs pp = p;
    pp.rows = g.rows;
    pp.K = g.W.K;
    TRY(qprep_row<MODE>(c, pp, *act));
    return gemm_tc<EPI>(c, g.W, *act, g.rows, g, ctas, split);
}

static mgb_status finalize(mgb_ctx *c, StaticState *st, int parts, int force) {
    const Config &g = c->cfg;
    const int threads = std::min(1024, std::max(32, 32 * st->b));
    if (st->sl >= 0) {  // --fast-vocab: source-token logits, then the concat argmax
        const mgb_ctx::Shortlist &sl = c->shortlists[st->sl];
        const size_t sh = (size_t)4 * g.d;
        cudaError_t e = allow_smem(src_logits_kernel, sh);
        const int sparts = (st->s + 7) / 8;  // source partials per row (8 positions a CTA)
        if (e == cudaSuccess)
            e = launch_pdl(src_logits_kernel, dim3(st->b, sparts), dim3(256), sh, c->stream, (const float *)st->x,
                           c->dec_norm.g, c->dec_norm.b, g.d, (const float *)st->src_emb, st->s, (int)sl.ids.size(),
                           st->src_v, st->src_i);
        ++c->launches;
        if (e != cudaSuccess) return cuda_err(e, "source logits launch");
        e = launch_pdl(greedy_finalize_sl_kernel, dim3(1), dim3(threads), 0, c->stream, (const float *)st->part_v,
                       (const uint32_t *)st->part_i, parts, st->b, (const float *)st->src_v,
                       (const uint32_t *)st->src_i, sparts, sl.d_ids, (int)sl.ids.size(),
                       (const uint32_t *)st->src_ids, st->s,
                       st->finished, st->ids, st->out, st->m, st->step, (uint32_t)g.eos, (uint32_t)g.pad, force);
        ++c->launches;
        return e == cudaSuccess ? MGB_OK : cuda_err(e, "finalize launch");
    }
    cudaError_t e = launch_pdl(greedy_finalize_kernel, dim3(1), dim3(threads), 0, c->stream,
                               (const float *)st->part_v, (const uint32_t *)st->part_i, parts, st->b,
                               st->finished, st->ids, st->out, st->m, st->step, (uint32_t)g.eos, (uint32_t)g.pad,
                               force);
    ++c->launches;
    if (e != cudaSuccess) return cuda_err(e, "finalize launch");
    return MGB_OK;
}

// ---------------------------------------------------------------------------
// Persistent step kernel (stepkernel.cuh): batches of at most 8 rows, the
// greedy step's f16 caches, quantized matrices.

static bool step_kernel_ok(const mgb_ctx *c, int b) {
    if (!c->step_kernel || b > kSmallRows) return false;
    const int hd = c->cfg.d / c->cfg.dec_heads;
    if (hd != 64 && hd != 128) return false;
    if (!tc_ok(c->embed)) return false;
    for (const DecLayer &L : c->dec)
        for (const Matrix *M : {&L.qkv, &L.out, &L.cq, &L.co, &L.up, &L.down}) {
            if (!tc_ok(*M)) return false;
            int r0, r1;
            cta_rows(M->Np, c->sms, 0, r0, r1);
            if (r1 - r0 > kStepRows) return false;  // the kernel stages at most kStepRows rows' bias / residual
        }
    return true;
}

// The state's phase table and shared-memory geometry (first use of a state).
static mgb_status build_step(mgb_ctx *c, StaticState *st) {
    if (st->phases) return MGB_OK;
    const Config &g = c->cfg;
    const int b = st->b, d = g.d, H = g.dec_heads, hd = d / H;
    const int NC = b <= 1 ? 1 : b <= 2 ? 2 : b <= 4 ? 4 : 8;
    std::vector<StepPhase> ph;
    int slot_bytes = 0;
    size_t act = 0;
    auto mm = [&](const Matrix &W, int epi, int mode, const float *x, const Norm *n, float *y, void *kc = nullptr,
                  void *vc = nullptr) {
        StepPhase p{};
        p.kind = PH_MM;
        p.W = W;
        p.epi = epi;
        p.mode = mode;
        p.x = x;
        if (n) {
            p.gamma = n->g;
            p.beta = n->b;
        }
        p.y = y;
        p.kc = kc;
        p.vc = vc;
        const int RB = row_bytes_of(W.type, W.K);
        const int per = (W.Np / 8 + c->sms - 1) / c->sms * 8;  // rows per CTA (stepkernel.cuh cta_rows)
        p.rsel = per > 8 && 32 * RB <= 36 * 1024 ? 4 : 1;
        slot_bytes = std::max(slot_bytes, 8 * p.rsel * RB);
        act = std::max(act, small_act_bytes(NC, W.K, W.type, mode));
        ph.push_back(p);
    };
    auto at = [&](bool self, int l) {
        StepPhase p{};
        p.kind = PH_ATTN;
        p.aq = st->q;
        p.K = self ? (const void *)st->kc[l] : (const void *)st->ck[l];
        p.V = self ? (const void *)st->vc[l] : (const void *)st->cv[l];
        p.kv_head = (long)(self ? st->m : st->s) * hd;
        p.kv_batch = (long)H * (self ? st->m : st->s) * hd;
        p.self = self;
        p.aout = st->a;
        ph.push_back(p);
    };
    for (int l = 0; l < g.dec_layers; ++l) {
        const DecLayer &L = c->dec[l];
        mm(L.qkv, EPI_QKV, l == 0 ? PREP_EMBED_LN : PREP_LN, st->x, &L.attn_norm, nullptr, st->kc[l], st->vc[l]);
        at(true, l);
        mm(L.out, EPI_RESID, PREP_PLAIN, st->a, nullptr, st->x);
        mm(L.cq, EPI_STORE, PREP_LN, st->x, &L.cross_norm, st->q);
        at(false, l);
        mm(L.co, EPI_RESID, PREP_PLAIN, st->a, nullptr, st->x);
        mm(L.up, EPI_RELU, PREP_LN, st->x, &L.ffn_norm, st->u);
        mm(L.down, EPI_RESID, PREP_PLAIN, st->u, nullptr, st->x);
    }
    slot_bytes = (slot_bytes + 127) / 128 * 128;
    act = (act + 127) / 128 * 128;
    const size_t escr = (size_t)8 * std::max(st->m, st->s) * 4;
    const int slots = (int)std::min<size_t>(8, (c->smem_optin - 8192 - act - escr) / slot_bytes);
    if (slots < 2) return set_err(MGB_ERR_UNSUPPORTED, "persistent step: shared memory");
    void *p = nullptr;
    TRY(c->dalloc(&p, sizeof(StepPhase) * ph.size()));
    st->allocs.push_back(p);
    st->phases = (StepPhase *)p;
    CK(cudaMemcpyAsync(st->phases, ph.data(), sizeof(StepPhase) * ph.size(), cudaMemcpyHostToDevice, c->stream));
    TRY(c->dalloc(&p, 256));
    st->allocs.push_back(p);
    st->bar = (uint32_t *)p;
    CK(cudaMemsetAsync(st->bar, 0, 256, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    if (!c->step_trace.empty()) {
        TRY(c->dalloc(&p, 8 * (8 * ph.size() + 1)));
        st->allocs.push_back(p);
        st->trace = (unsigned long long *)p;
        CK(cudaMemset(st->trace, 0, 8 * (8 * ph.size() + 1)));
        st->phase_host = ph;
        st->trace_path = c->step_trace;
    }
    st->nphases = (int)ph.size();
    st->step_slots = slots;
    st->step_ctas = c->sms;
    st->step_slot_bytes = slot_bytes;
    st->step_act_bytes = (int)act;
    st->step_smem = (size_t)slots * slot_bytes + act + escr;
    return MGB_OK;
}

template <int NC, int NW>
static cudaError_t step_launch(mgb_ctx *c, const StepArgs &a, size_t smem) {
    auto kern = step_kernel<NC, NW>;
    cudaError_t e = allow_smem(kern, smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(c->sms);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = c->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: the grid barriers need it
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, a);
}

// The decoder layers of a greedy step as one persistent launch (stepkernel.cuh).
static mgb_status launch_step_persistent(mgb_ctx *c, StaticState *st) {
    TRY(build_step(c, st));
    const Config &g = c->cfg;
    StepArgs a{};
    a.ph = st->phases;
    a.nph = st->nphases;
    a.rows = st->b;
    a.H = g.dec_heads;
    a.hd = g.d / g.dec_heads;
    a.m = st->m;
    a.max_keys = std::max(st->m, st->s);
    a.kv_f32 = 0;
    a.lens = st->lens;
    a.embed = c->embed;
    a.ids = st->ids;
    a.step = st->step;
    a.pos_table = c->pos;
    a.pos_base = (uint32_t)g.pad + 1;
    a.scale = c->embed_scale;
    a.x = st->x;
    a.q = st->q;
    a.bar = st->bar;
    a.abort_flag = st->bar + 32;
    a.err = c->d_err;
    a.wait_ns = c->test_wait_ns;
    a.withhold = c->test_withhold_step;
    a.trace = st->trace;
    a.slots = st->step_slots;
    a.slot_bytes = st->step_slot_bytes;
    a.act_bytes = st->step_act_bytes;
    CK(cudaMemsetAsync(st->bar, 0, 256, c->stream));
    cudaError_t e;
    switch (st->b <= 1 ? 1 : st->b <= 2 ? 2 : st->b <= 4 ? 4 : 8) {
        case 1: e = step_launch<1, 4>(c, a, st->step_smem); break;
        case 2: e = step_launch<2, 4>(c, a, st->step_smem); break;
        case 4: e = step_launch<4, 4>(c, a, st->step_smem); break;
        default: e = step_launch<8, 2>(c, a, st->step_smem); break;
    }
    ++c->launches;
    return e == cudaSuccess ? MGB_OK : cuda_err(e, "persistent step launch");
}

// How a decoder step runs: the K/V element type and the rows of the
// reference's matmul calls (candle picks MMVQ or MMQ, and MMVQ's warp count,
// from them).
struct StepMode {
    bool kv32 = false;  // the generic decode's f32 self / cross K/V (beam search, model.rs:124-133)
    int cls = 0;        // rows of the decoder-layer matmul calls (0: the state's rows)
    int lm_cls = 0;     // rows of the LM head call (0: the state's rows)
    bool lm = true;     // run the LM head (a prefill position whose logits are not used has none)
};

// One decoder step on the state's fixed buffers (model.rs:552-612):
// per layer fused QKV (+ K/V cache write), self-attention, out-proj +
// residual, cross-q, cross-attention, cross-out + residual, FFN up + ReLU,
// down + residual, every LayerNorm folded into the next matmul's activation
// prologue; then the tied LM head fused with the first argmax pass, finalize.
// Calls of up to 8 rows run the small-batch kernel (MMVQ); larger ones the
// tensor-core kernel (MMQ), which reads q8_1 activations that qprep_row, or for
// the out projections the attention kernel itself, writes.
static mgb_status launch_step(mgb_ctx *c, StaticState *st, float *logits, int force,
                              cudaEvent_t lm0 = nullptr, cudaEvent_t lm1 = nullptr, bool finalize_step = true,
                              const StepMode &mode = StepMode{}) {
    const Config &g = c->cfg;
    const int b = st->b, d = g.d, H = g.dec_heads, hd = d / H;
    // the decoder layers of a small greedy batch: one persistent launch
    const bool persistent = !mode.kv32 && !mode.cls && !mode.lm_cls && step_kernel_ok(c, b);
    const int cls = mode.cls ? mode.cls : b, lm_cls = mode.lm_cls ? mode.lm_cls : b;
    const bool tc = cls > kSmallRows && tc_ok(c->dec[0].qkv);
    const SplitBufs *sp = tc && c->tc_split && st->split.part ? &st->split : nullptr;
    const bool kv32 = mode.kv32;
    QAct *X = &st->act;  // tensor-core activations of the next matmul
    // attention whose outputs also go, as q8_1, into the next matmul's input
    const bool attn_q = tc && hd % 32 == 0;
    auto attn = [&](const AttnArgs &a) { return kv32 ? attend<float>(c, a) : attend<__half>(c, a); };
    if (persistent) TRY(launch_step_persistent(c, st));
    for (int l = 0; l < g.dec_layers && !persistent; ++l) {
        const DecLayer &L = c->dec[l];
        // attn_norm(x) (layer 0: x = E[id]*scale + pos) -> fused QKV -> q, K/V cache slot *step
        GemvArgs gq = mm_out(L.qkv, b);
        gq.q = st->q;
        gq.kc = kv32 ? (void *)st->kc32[l] : (void *)st->kc[l];
        gq.vc = kv32 ? (void *)st->vc32[l] : (void *)st->vc[l];
        gq.kv_f32 = kv32;
        gq.step = st->step;
        gq.H = H;
        gq.hd = hd;
        gq.m = st->m;
        PrepArgs pq = prep_src(st->x, &L.attn_norm);
        if (l == 0) {
            pq.x_out = st->x;
            pq.embed = c->embed;
            pq.ids = st->ids;
            pq.step = st->step;
            pq.pos_table = c->pos;
            pq.pos_base = (uint32_t)g.pad + 1;
            pq.scale = c->embed_scale;
            TRY((matmul<EPI_QKV, PREP_EMBED_LN>(c, gq, pq, X, nullptr, sp, cls)));
        } else {
            TRY((matmul<EPI_QKV, PREP_LN>(c, gq, pq, X, nullptr, sp, cls)));
        }
        AttnArgs sa{};
        sa.q = st->q;
        sa.q_row = d;
        sa.K = gq.kc;
        sa.V = gq.vc;
        sa.kv_row = hd;
        sa.kv_head = (long)st->m * hd;
        sa.kv_batch = (long)H * st->m * hd;
        sa.step = st->step;
        sa.out = st->a;
        sa.out_row = d;
        sa.H = H;
        sa.hd = hd;
        sa.rows = b;
        sa.queries = 1;
        sa.max_keys = st->m;
        if (attn_q) sa.qo = *X;
        TRY(attn(sa));
        GemvArgs go = mm_out(L.out, b);
        go.y = st->x;
        if (attn_q) TRY(gemm_tc<EPI_RESID>(c, L.out, *X, b, go, nullptr, sp));
        else TRY((matmul<EPI_RESID, PREP_PLAIN>(c, go, prep_src(st->a, nullptr), X, nullptr, sp, cls)));
        // cross_norm -> cross_q -> cross attention -> cross_out + residual
        GemvArgs gc = mm_out(L.cq, b);
        gc.y = st->q;
        TRY((matmul<EPI_STORE, PREP_LN>(c, gc, prep_src(st->x, &L.cross_norm), X, nullptr, sp, cls)));
        AttnArgs ca = sa;
        ca.K = kv32 ? (const void *)st->ck32[l] : (const void *)st->ck[l];
        ca.V = kv32 ? (const void *)st->cv32[l] : (const void *)st->cv[l];
        ca.kv_head = (long)st->s * hd;
        ca.kv_batch = (long)H * st->s * hd;
        ca.step = nullptr;
        ca.lens = st->lens;
        ca.max_keys = st->s;
        TRY(attn(ca));
        GemvArgs gco = mm_out(L.co, b);
        gco.y = st->x;
        if (attn_q) TRY(gemm_tc<EPI_RESID>(c, L.co, *X, b, gco, nullptr, sp));
        else TRY((matmul<EPI_RESID, PREP_PLAIN>(c, gco, prep_src(st->a, nullptr), X, nullptr, sp, cls)));
        // ffn_norm -> up + ReLU -> down + residual
        GemvArgs gu = mm_out(L.up, b);
        gu.y = st->u;
        GemvArgs gd = mm_out(L.down, b);
        gd.y = st->x;
        // tensor-core path: the up epilogue writes the down matmul's q8_1
        // activations itself (into a second buffer: the up matmul reads X)
        const bool hq = c->ffn_q8 && tc && tc_ok(L.up) && tc_ok(L.down) && L.up.N % 128 == 0 && st->act2.tq;
        if (hq) gu.qo = st->act2;
        TRY((matmul<EPI_RELU, PREP_LN>(c, gu, prep_src(st->x, &L.ffn_norm), X, nullptr, sp, cls)));
        if (hq) TRY(gemm_tc<EPI_RESID>(c, L.down, st->act2, b, gd, nullptr, sp));
        else TRY((matmul<EPI_RESID, PREP_PLAIN>(c, gd, prep_src(st->u, nullptr), X, nullptr, sp, cls)));
    }
    if (!mode.lm) return MGB_OK;
    // dec_norm -> tied LM head (or the shortlist's reduced head) fused with the
    // first argmax pass -> greedy bookkeeping
    GemvArgs gl = mm_out(st->sl >= 0 ? c->shortlists[st->sl].W : c->embed, b);
    gl.part_v = st->part_v;
    gl.part_i = st->part_i;
    gl.logits = logits;
    if (lm0) CK(cudaEventRecord(lm0, c->stream));
    int parts = kLmParts;
    TRY((matmul<EPI_ARGMAX, PREP_LN>(c, gl, prep_src(st->x, &c->dec_norm), X, &parts, nullptr, lm_cls)));
    st->lm_parts = parts;
    if (lm1) CK(cudaEventRecord(lm1, c->stream));
    if (!finalize_step) return MGB_OK;
    return finalize(c, st, parts, force);
}

// ---------------------------------------------------------------------------
// Encoder (model.rs:463-500)

// A batch's device buffer of at least `bytes`: the smallest pooled buffer that
// fits, else a new allocation.
static mgb_status batch_buf(mgb_ctx *c, size_t bytes, mgb_batch *B) {
    int best = -1;
    for (size_t i = 0; i < c->batch_pool.size(); ++i)
        if (c->batch_pool[i].bytes >= bytes && (best < 0 || c->batch_pool[i].bytes < c->batch_pool[best].bytes))
            best = (int)i;
    if (best >= 0) {
        B->buf = c->batch_pool[best].p;
        B->buf_bytes = c->batch_pool[best].bytes;
        c->batch_pool_bytes -= B->buf_bytes;
        c->batch_pool.erase(c->batch_pool.begin() + best);
        return MGB_OK;
    }
    TRY(c->dalloc(&B->buf, bytes));
    B->buf_bytes = bytes;
    return MGB_OK;
}

// Back to the pool (work queued on the context's stream that still reads the
// buffer runs before any later use of it, which is queued on the same stream).
static void batch_release(mgb_ctx *c, mgb_batch *B) {
    if (!B->buf) return;
    if (c->batch_pool_bytes + B->buf_bytes <= kBatchPoolBytes) {
        c->batch_pool.push_back({B->buf, B->buf_bytes});
        c->batch_pool_bytes += B->buf_bytes;
    } else {
        cudaFree(B->buf);
    }
    B->buf = nullptr;
    B->cross = nullptr;
    B->d_lens = nullptr;
}

// ids: [b][S] right-padded, S = the longest sentence (pad_batch, model.rs:480-500;
// the matmuls then see b*S rows, as the reference's).
static mgb_status encode(mgb_ctx *c, const uint32_t *ids, const uint32_t *lens, int b, int S, mgb_batch **out) {
    const Config &g = c->cfg;
    const int d = g.d, H = g.enc_heads, hd = d / H, rows = b * S, ffn = g.enc_ffn, kmax = std::max(d, ffn);
    uint32_t *d_ids, *d_lens;
    float *x, *qkv, *a, *u;
    QAct act;
    // temporaries carved from the context's encoder workspace (grown, never
    // shrunk, released by mgb_clear_cache / mgb_close): no allocation per call
    {
        const int rp = (rows + 63) / 64 * 64, nbm = kmax / 32;
        const size_t sz[] = {(size_t)4 * rows, (size_t)4 * b, (size_t)4 * rows * d, (size_t)4 * rows * 3 * d,
                             (size_t)4 * rows * d, (size_t)4 * rows * ffn, (size_t)nbm * rp * 32, (size_t)nbm * rp * 8};
        constexpr int NP = sizeof sz / sizeof sz[0];
        size_t total = 0;
        for (size_t n : sz) total += (n + 255) / 256 * 256;
        if (total > c->enc_ws_bytes) {
            if (c->enc_ws) cudaFree(c->enc_ws);
            c->enc_ws = nullptr;
            c->enc_ws_bytes = 0;
            TRY(c->dalloc(&c->enc_ws, total));
            c->enc_ws_bytes = total;
        }
        uint8_t *w = reinterpret_cast<uint8_t *>(c->enc_ws);
        void *ptrs[NP];
        for (int i = 0; i < NP; ++i) {
            ptrs[i] = w;
            w += (sz[i] + 255) / 256 * 256;
        }
        d_ids = (uint32_t *)ptrs[0];
        d_lens = (uint32_t *)ptrs[1];
        x = (float *)ptrs[2];
        qkv = (float *)ptrs[3];
        a = (float *)ptrs[4];
        u = (float *)ptrs[5];
        act.tq = (uint8_t *)ptrs[6];
        act.trec = (float2 *)ptrs[7];
        act.rs = rp;
    }
    CK(cudaMemcpyAsync(d_ids, ids, (size_t)4 * rows, cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemcpyAsync(d_lens, lens, (size_t)4 * b, cudaMemcpyHostToDevice, c->stream));
    TRY(launch_check(c, [&] {
        embed_tokens_kernel<<<(rows + 7) / 8, 256, 0, c->stream>>>(c->embed, d_ids, d_lens, S, rows, c->pos,
                                                                   (uint32_t)g.pad, c->embed_scale, x);
    }));
    for (int l = 0; l < g.enc_layers; ++l) {
        const EncLayer &L = c->enc[l];
        GemvArgs gq = mm_out(L.qkv, rows);
        gq.y = qkv;
        TRY((matmul<EPI_STORE, PREP_LN>(c, gq, prep_src(x, &L.attn_norm), &act)));
        AttnArgs at{};
        at.q = qkv;
        at.q_row = 3 * d;
        at.K = qkv + d;
        at.V = qkv + 2 * d;
        at.kv_row = 3 * d;
        at.kv_head = hd;
        at.kv_batch = (long)S * 3 * d;
        at.lens = d_lens;
        at.out = a;
        at.out_row = d;
        at.H = H;
        at.hd = hd;
        at.rows = b;
        at.queries = S;
        at.max_keys = S;
        TRY(attend<float>(c, at));
        GemvArgs go = mm_out(L.out, rows);
        go.y = x;
        TRY((matmul<EPI_RESID, PREP_PLAIN>(c, go, prep_src(a, nullptr), &act)));
        GemvArgs gu = mm_out(L.up, rows);
        gu.y = u;
        TRY((matmul<EPI_RELU, PREP_LN>(c, gu, prep_src(x, &L.ffn_norm), &act)));
        GemvArgs gd = mm_out(L.down, rows);
        gd.y = x;
        TRY((matmul<EPI_RESID, PREP_PLAIN>(c, gd, prep_src(u, nullptr), &act)));
    }
    auto B = std::make_unique<mgb_batch>();
    B->b = b;
    B->s = S;
    B->owner = c;
    B->lens.assign(lens, lens + b);
    B->src.assign(ids, ids + (size_t)b * S);
    const int Hd = g.dec_heads, hdd = d / Hd;
    const size_t per = (size_t)b * Hd * S * hdd;
    B->cross_bytes = per * 4 * 2 * g.dec_layers;
    TRY(batch_buf(c, (B->cross_bytes + 255) / 256 * 256 + (size_t)4 * b, B.get()));
    B->cross = (float *)B->buf;
    B->d_lens = (uint32_t *)((uint8_t *)B->buf + (B->cross_bytes + 255) / 256 * 256);
    mgb_status s = MGB_OK;
    CK(cudaMemcpyAsync(B->d_lens, lens, (size_t)4 * b, cudaMemcpyHostToDevice, c->stream));
    // enc_norm(x) is the input of every decoder layer's cross K/V projection
    // (model.rs:471-475); its q8_1 activations are prepared once
    const PrepArgs pn = prep_src(x, &c->enc_norm);
    const bool tc = rows > kSmallRows && tc_ok(c->dec[0].ckv);
    if (tc) {
        PrepArgs pp = pn;
        pp.rows = rows;
        pp.K = d;
        s = qprep_row<PREP_LN>(c, pp, act);
    }
    for (int l = 0; l < g.dec_layers && s == MGB_OK; ++l) {
        GemvArgs gk = mm_out(c->dec[l].ckv, rows);
        gk.kc = B->cross + per * (2 * l);
        gk.vc = B->cross + per * (2 * l + 1);
        gk.H = Hd;
        gk.hd = hdd;
        gk.S = S;
        s = tc && tc_ok(c->dec[l].ckv) ? gemm_tc<EPI_CROSSKV>(c, c->dec[l].ckv, act, rows, gk)
                                       : small_mm<EPI_CROSSKV, PREP_LN>(c, gk, pn);
    }
    if (s != MGB_OK) {
        batch_release(c, B.get());
        return s;
    }
    uint32_t derr = 0;
    CK(cudaMemcpyAsync(&derr, c->d_err, 4, cudaMemcpyDeviceToHost, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    if (derr) {
        cudaMemsetAsync(c->d_err, 0, 4, c->stream);
        batch_release(c, B.get());
        return set_err(MGB_ERR_CUDA, "a device-side wait ran out of time in the encoder (flags %u)", derr);
    }
    c->batches.insert(B.get());
    *out = B.release();
    return MGB_OK;
}

// ---------------------------------------------------------------------------
// Greedy decoding with the graph cache (graph.rs:204-298)

static void evict(mgb_ctx *c, StaticState *keep) {
    bool dropped_graph = false;
    for (;;) {
        size_t total = kGraphBytes;
        for (auto &e : c->cache) total += e->bytes + (e->exec ? kGraphBytes : 0);
        if (total <= c->opts.graph_cache_bytes || c->cache.size() <= 1) break;
        int victim = -1;
        for (size_t i = 0; i < c->cache.size(); ++i)
            if (c->cache[i].get() != keep && (victim < 0 || c->cache[i]->last_used < c->cache[victim]->last_used))
                victim = (int)i;
        if (victim < 0) break;
        dropped_graph |= c->cache[victim]->exec != nullptr;
        free_state(c->cache[victim].get());
        c->cache.erase(c->cache.begin() + victim);
    }
    if (dropped_graph) cudaDeviceGraphMemTrim(c->device);
}

static void clear_cache(mgb_ctx *c) {
    cudaStreamSynchronize(c->stream);
    for (auto &e : c->cache) free_state(e.get());
    c->cache.clear();
    if (c->enc_ws) cudaFree(c->enc_ws);
    c->enc_ws = nullptr;
    c->enc_ws_bytes = 0;
    for (const PoolBuf &e : c->batch_pool) cudaFree(e.p);
    c->batch_pool.clear();
    c->batch_pool_bytes = 0;
    cudaDeviceGraphMemTrim(c->device);
}

static mgb_status set_ids(mgb_ctx *c, StaticState *st, uint32_t id) {
    std::vector<uint32_t> v(st->b, id);
    CK(cudaMemcpyAsync(st->ids, v.data(), 4 * st->b, cudaMemcpyHostToDevice, c->stream));
    return cudaStreamSynchronize(c->stream) == cudaSuccess ? MGB_OK : cuda_err(cudaGetLastError(), "set_ids");
}

static mgb_status reset_finished(mgb_ctx *c, StaticState *st, int active) {
    std::vector<uint8_t> f(st->b);
    for (int i = 0; i < st->b; ++i) f[i] = i >= active;
    CK(cudaMemcpyAsync(st->finished, f.data(), st->b, cudaMemcpyHostToDevice, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    return MGB_OK;
}

// Finds or creates the static state of the (rows, source, output) bucket and
// loads the batch into it (graph.rs:236-268).
// rep > 1: every sentence fills rep consecutive rows (beam search).
static mgb_status acquire_state(mgb_ctx *c, const mgb_batch *B, int max_new, bool pad_rows, StaticState **out,
                                int rep = 1, int sl = -1) {
    const Config &g = c->cfg;
    const int n = B->b * rep, H = g.dec_heads, hd = g.d / H;
    const int b = pad_rows ? (int)next_pow2((uint32_t)n) : n;
    if (b > 128) return set_err(MGB_ERR_INVALID, "batch of %d rows exceeds 128", n);
    const int s = bucket(B->s, 16, g.max_pos), m = bucket(max_new + 2, 32, g.max_pos);
    StaticState *st = nullptr;
    for (auto &e : c->cache)
        if (e->b == b && e->s == s && e->m == m && e->sl == sl) st = e.get();  // (graph.rs:243 key)
    if (!st) {
        TRY(new_state(c, b, s, m, &st));
        c->cache.emplace_back(st);
        if (sl >= 0) {
            st->sl = sl;
            for (void **p : {(void **)&st->src_ids, (void **)&st->src_v, (void **)&st->src_i, (void **)&st->src_emb}) {
                // ids [b][s]; partials [b][ceil(s / 8)]; embeddings [b][s][d]
                const size_t n = (size_t)4 * b * s * (p == (void **)&st->src_emb ? g.d : 1);
                TRY(c->dalloc(p, n));
                st->allocs.push_back(*p);
                st->bytes += n;
            }
        }
        evict(c, st);
    }
    st->last_used = ++c->clock;
    // reset (graph.rs:91-113): cross K/V (converted to f16, graph.rs:95-96), lens,
    // start token, step, finished
    const size_t per = (size_t)B->b * H * B->s * hd;
    for (int l = 0; l < g.dec_layers; ++l) {
        TRY(launch_check(c, [&] {
            cross_load_kernel<<<c->sms * 4, 256, 0, c->stream>>>(B->cross + per * 2 * l, st->ck[l], 1, n, rep, H, B->s,
                                                                 s, hd);
            cross_load_kernel<<<c->sms * 4, 256, 0, c->stream>>>(B->cross + per * (2 * l + 1), st->cv[l], 1, n, rep,
                                                                 H, B->s, s, hd);
        }));
    }
    if (sl >= 0) {  // source ids of every row, pad past its length (graph.rs:98-105)
        std::vector<uint32_t> ids((size_t)b * s, (uint32_t)g.pad);
        for (int i = 0; i < n; ++i)
            for (int j = 0; j < (int)B->lens[i / rep] && j < s; ++j) ids[(size_t)i * s + j] = B->src[(size_t)(i / rep) * B->s + j];
        CK(cudaMemcpyAsync(st->src_ids, ids.data(), 4 * ids.size(), cudaMemcpyHostToDevice, c->stream));
        TRY(launch_check(c, [&] {
            src_embed_kernel<<<c->sms * 4, 256, 0, c->stream>>>(c->embed, st->src_ids, b * s, g.d, st->src_emb);
        }));
        CK(cudaStreamSynchronize(c->stream));
    }
    std::vector<uint32_t> lens(b, 1);
    for (int i = 0; i < n; ++i) lens[i] = B->lens[i / rep];
    CK(cudaMemcpyAsync(st->lens, lens.data(), 4 * b, cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemsetAsync(st->step, 0, 4, c->stream));
    if (st->split.count) CK(cudaMemsetAsync(st->split.count, 0, 4 * 4096, c->stream));
    TRY(set_ids(c, st, (uint32_t)g.start));
    TRY(reset_finished(c, st, n));
    *out = st;
    return MGB_OK;
}

// Beam-search buffers of a state (first use).
static mgb_status ensure_beam(mgb_ctx *c, StaticState *st) {
    if (st->beam_logits) return MGB_OK;
    const Config &g = c->cfg;
    const int b = st->b, H = g.dec_heads, hd = g.d / H;
    auto A = [&](void **p, size_t n) -> mgb_status {
        TRY(c->dalloc(p, n));
        st->allocs.push_back(*p);
        st->bytes += n;
        return MGB_OK;
    };
    // + 16 bytes: the top-k kernel's bulk copies round a row's end up to 16 bytes
    TRY(A((void **)&st->beam_logits, (size_t)4 * b * g.V + 16));
    TRY(A((void **)&st->beam_vals, (size_t)4 * b * 8));
    TRY(A((void **)&st->beam_idx, (size_t)4 * b * 8));
    TRY(A((void **)&st->beam_from, (size_t)4 * b));
    for (auto *v : {&st->kc32, &st->vc32, &st->kc32b, &st->vc32b, &st->ck32, &st->cv32}) v->resize(g.dec_layers);
    for (int l = 0; l < g.dec_layers; ++l) {
        for (auto *v : {&st->kc32, &st->vc32, &st->kc32b, &st->vc32b})
            TRY(A((void **)&(*v)[l], (size_t)4 * b * H * st->m * hd));
        TRY(A((void **)&st->ck32[l], (size_t)4 * b * H * st->s * hd));
        TRY(A((void **)&st->cv32[l], (size_t)4 * b * H * st->s * hd));
    }
    return MGB_OK;
}

// Log-softmax statistics and top-k of rows of logits on the device
// (beam_topk_kernel). `logits` holds rows x V floats and at least 16 bytes
// more (the kernel's bulk copies round a row's end up to 16 bytes).
template <int K>
static mgb_status beam_topk_k(mgb_ctx *c, const float *logits, int rows, int V, float *vals, uint32_t *idx) {
    cudaError_t e = allow_smem(beam_topk_kernel<K>, kTopkSmem);
    if (e == cudaSuccess) {
        beam_topk_kernel<K><<<rows, kTopkThreads, kTopkSmem, c->stream>>>(logits, V, vals, idx, c->d_err,
                                                                           c->test_wait_ns, c->test_withhold_topk);
        e = cudaGetLastError();
    }
    ++c->launches;
    return e == cudaSuccess ? MGB_OK : cuda_err(e, "top-k launch");
}

static mgb_status beam_topk(mgb_ctx *c, const float *logits, int rows, int V, int k, float *vals, uint32_t *idx) {
    switch (k) {
        case 1: return beam_topk_k<1>(c, logits, rows, V, vals, idx);
        case 2: return beam_topk_k<2>(c, logits, rows, V, vals, idx);
        case 3: return beam_topk_k<3>(c, logits, rows, V, vals, idx);
        case 4: return beam_topk_k<4>(c, logits, rows, V, vals, idx);
        case 5: return beam_topk_k<5>(c, logits, rows, V, vals, idx);
        case 6: return beam_topk_k<6>(c, logits, rows, V, vals, idx);
        case 7: return beam_topk_k<7>(c, logits, rows, V, vals, idx);
        default: return beam_topk_k<8>(c, logits, rows, V, vals, idx);
    }
}

// Rust's f32::total_cmp key (IEEE total order as a signed integer).
static int32_t total_key(float f) {
    int32_t v;
    memcpy(&v, &f, 4);
    return v ^ (int32_t)(((uint32_t)(v >> 31)) >> 1);
}

// Beam search (translator.rs:250-335; top-k 343-358) with the reference's
// generic decode (Nllb::decode, model.rs:515-540): rows = sentences x k on the
// device with f32 self and cross K/V (KvCache, model.rs:124-133); the prefill
// [</s>, tgt] is one call of 2 tokens per row in the reference (its matmuls see
// 2*rows rows, its LM head rows rows), run here as two single-token passes with
// that row class -- each output of those matmuls depends only on its own row and
// the class, so the values are the same; per step the LM head writes every
// row's logits, the device computes log_softmax statistics and each row's top
// k, the host merges the k*k candidates of every sentence (score descending,
// ties in insertion order, beam-major then rank), retires hypotheses that end in
// eos or at max_new with score / (len+1)^lp, and the self-attention caches are
// gathered by source row (DecoderState::reorder; a row's cross K/V stays its
// sentence's).
static mgb_status run_beam(mgb_ctx *c, const mgb_batch *B, uint32_t tgt, int k, float lp, int max_new,
                           uint32_t *out_ids, uint32_t *out_lens) {
    const Config &g = c->cfg;
    const int nb = B->b, rows = nb * k, V = g.V, H = g.dec_heads, hd = g.d / H;
    const uint32_t eos = (uint32_t)g.eos;
    StaticState *st = nullptr;
    TRY(acquire_state(c, B, max_new, false, &st, k));
    TRY(ensure_beam(c, st));
    const size_t per = (size_t)B->b * H * B->s * hd;
    for (int l = 0; l < g.dec_layers; ++l) {
        TRY(launch_check(c, [&] {
            cross_load_kernel<<<c->sms * 4, 256, 0, c->stream>>>(B->cross + per * 2 * l, st->ck32[l], 0, rows, k, H,
                                                                 B->s, st->s, hd);
            cross_load_kernel<<<c->sms * 4, 256, 0, c->stream>>>(B->cross + per * (2 * l + 1), st->cv32[l], 0, rows,
                                                                 k, H, B->s, st->s, hd);
        }));
    }
    auto set_step = [&](uint32_t v) -> mgb_status {
        CK(cudaMemcpyAsync(st->step, &v, 4, cudaMemcpyHostToDevice, c->stream));
        return cudaStreamSynchronize(c->stream) == cudaSuccess ? MGB_OK : cuda_err(cudaGetLastError(), "beam step");
    };
    StepMode prefill0, prefill1, stepm;
    prefill0.kv32 = prefill1.kv32 = stepm.kv32 = true;
    prefill0.cls = prefill1.cls = 2 * rows;
    prefill0.lm = false;  // the first position's logits are not used (model.rs:535)
    TRY(set_step(0));
    TRY(launch_step(c, st, nullptr, 1, nullptr, nullptr, false, prefill0));
    TRY(set_ids(c, st, tgt));
    TRY(set_step(1));
    TRY(launch_step(c, st, st->beam_logits, 1, nullptr, nullptr, false, prefill1));
    const int L = max_new + 1;
    std::vector<float> alive_score(rows, 0.0f), nscore(rows), vals((size_t)rows * k);
    std::vector<uint32_t> alive_tok((size_t)rows * L, 0), ntok((size_t)rows * L, 0), idx((size_t)rows * k);
    std::vector<int> alive_len(rows, 0), nlen(rows), n_alive(nb, 1), reorder(rows);
    std::vector<uint32_t> next(rows);
    struct Done {
        float score;
        std::vector<uint32_t> tok;
    };
    std::vector<std::vector<Done>> done(nb);
    std::vector<uint8_t> is_done(nb, 0);
    const size_t cap_done = (size_t)4 * k * L;
    struct Cand {
        float score;
        int beam;
        uint32_t tok;
    };
    std::vector<Cand> cands((size_t)k * k);
    for (int step = 1; step <= max_new; ++step) {
        TRY(beam_topk(c, st->beam_logits, rows, V, k, st->beam_vals, st->beam_idx));
        CK(cudaMemcpyAsync(vals.data(), st->beam_vals, 4 * vals.size(), cudaMemcpyDeviceToHost, c->stream));
        CK(cudaMemcpyAsync(idx.data(), st->beam_idx, 4 * idx.size(), cudaMemcpyDeviceToHost, c->stream));
        CK(cudaStreamSynchronize(c->stream));
        int nr = 0;
        for (int s = 0; s < nb; ++s) {
            int nc = 0;
            for (int bi = 0; bi < n_alive[s]; ++bi) {
                const int row = s * k + bi;
                for (int j = 0; j < k; ++j)
                    cands[nc++] = {alive_score[row] + vals[(size_t)row * k + j], bi, idx[(size_t)row * k + j]};
            }
            // stable sort, descending by total order
            for (int i = 1; i < nc; ++i) {
                const Cand t = cands[i];
                int q = i - 1;
                while (q >= 0 && total_key(t.score) > total_key(cands[q].score)) {
                    cands[q + 1] = cands[q];
                    --q;
                }
                cands[q + 1] = t;
            }
            int na = 0;
            for (int ci = 0; ci < nc && na < k; ++ci) {
                const Cand &cd = cands[ci];
                const int src = s * k + cd.beam;
                if (cd.tok == eos || step == max_new) {
                    if (!is_done[s] && done[s].size() < cap_done) {
                        Done dn;
                        dn.tok.assign(alive_tok.begin() + (size_t)src * L, alive_tok.begin() + (size_t)src * L + alive_len[src]);
                        if (cd.tok != eos) dn.tok.push_back(cd.tok);
                        const int dl = (int)dn.tok.size();
                        const float pen = powf((float)(dl + 1 > 1 ? dl + 1 : 1), lp);
                        dn.score = cd.score / pen;
                        done[s].push_back(std::move(dn));
                    }
                    continue;
                }
                const int dst = s * k + na;
                std::copy(alive_tok.begin() + (size_t)src * L, alive_tok.begin() + (size_t)src * L + alive_len[src],
                          ntok.begin() + (size_t)dst * L);
                ntok[(size_t)dst * L + alive_len[src]] = cd.tok;
                nlen[dst] = alive_len[src] + 1;
                nscore[dst] = cd.score;
                reorder[nr] = src;
                next[nr] = cd.tok;
                ++nr;
                ++na;
            }
            float best_done = -INFINITY;
            for (const Done &dn : done[s]) best_done = std::max(best_done, dn.score);
            const float best_alive = na > 0 ? nscore[s * k] / powf((float)(step + 1), lp) : -INFINITY;
            if ((int)done[s].size() >= k && best_done >= best_alive) is_done[s] = 1;
            while (na < k) {
                const int dst = s * k + na;
                reorder[nr] = s * k;
                next[nr] = eos;
                ++nr;
                nscore[dst] = -INFINITY;
                nlen[dst] = 0;
                ++na;
            }
            n_alive[s] = k;
        }
        alive_score = nscore;
        alive_tok = ntok;
        alive_len = nlen;
        bool all = true;
        for (int s = 0; s < nb; ++s) all = all && is_done[s];
        if (step == max_new || all) break;
        // reorder the self-attention caches (positions 0..step) by source row
        CK(cudaMemcpyAsync(st->beam_from, reorder.data(), 4 * rows, cudaMemcpyHostToDevice, c->stream));
        CK(cudaMemcpyAsync(st->ids, next.data(), 4 * rows, cudaMemcpyHostToDevice, c->stream));
        for (int l0 = 0; l0 < g.dec_layers; l0 += 64) {
            KvGather kg{};
            kg.n = 0;
            for (int l = l0; l < std::min(g.dec_layers, l0 + 64); ++l) {
                kg.src[kg.n] = st->kc32[l];
                kg.dst[kg.n++] = st->kc32b[l];
                kg.src[kg.n] = st->vc32[l];
                kg.dst[kg.n++] = st->vc32b[l];
            }
            TRY(launch_check(c, [&] {
                kv_gather_kernel<<<c->sms * 4, 256, 0, c->stream>>>(kg, st->beam_from, rows, H, st->m, hd, step + 1, 4);
            }));
        }
        std::swap(st->kc32, st->kc32b);
        std::swap(st->vc32, st->vc32b);
        TRY(set_step((uint32_t)step + 1));
        TRY(launch_step(c, st, st->beam_logits, 1, nullptr, nullptr, false, stepm));
    }
    uint32_t derr = 0;
    CK(cudaMemcpyAsync(&derr, c->d_err, 4, cudaMemcpyDeviceToHost, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    if (derr) {
        cudaMemsetAsync(c->d_err, 0, 4, c->stream);
        return set_err(MGB_ERR_CUDA, "a device-side wait ran out of time (flags %u)", derr);
    }
    for (int s = 0; s < nb; ++s) {
        const uint32_t *tok = nullptr;
        int len = 0;
        if (!done[s].empty()) {
            int best = -1;
            float bs = -INFINITY;
            for (int q = 0; q < (int)done[s].size(); ++q)
                if (best < 0 || done[s][q].score >= bs) {  // max_by: the last maximum wins
                    bs = done[s][q].score;
                    best = q;
                }
            tok = done[s][best].tok.data();
            len = (int)done[s][best].tok.size();
        } else {
            int best = -1;
            float bs = -INFINITY;
            for (int bi = 0; bi < k; ++bi)
                if (best < 0 || alive_score[s * k + bi] >= bs) {
                    bs = alive_score[s * k + bi];
                    best = bi;
                }
            tok = alive_tok.data() + (size_t)(s * k + best) * L;
            len = alive_len[s * k + best];
        }
        if (out_lens) out_lens[s] = (uint32_t)len;
        for (int t = 0; t < max_new; ++t) out_ids[(size_t)s * max_new + t] = t < len ? tok[t] : (uint32_t)g.pad;
    }
    return MGB_OK;
}

static mgb_status run_greedy(mgb_ctx *c, const mgb_batch *B, uint32_t tgt, int max_new, int sync_every, int force,
                             uint32_t *out_ids, uint32_t *out_lens, float *logits_host, int sl = -1) {
    const Config &g = c->cfg;
    const int n = B->b;
    const bool capture = c->capture && c->opts.use_graphs && !logits_host;
    StaticState *st = nullptr;
    TRY(acquire_state(c, B, max_new, capture, &st, 1, sl));
    const int b = st->b, m = st->m;
    float *d_logits = nullptr;
    if (logits_host) {
        if (!st->logits) {
            void *p;
            TRY(c->dalloc(&p, (size_t)4 * b * g.V));
            st->logits = (float *)p;
            st->allocs.push_back(p);
        }
        d_logits = st->logits;
    }
    // Step 0 consumes decoder_start; its output is replaced by the forced language token.
    TRY(launch_step(c, st, nullptr, force));
    TRY(set_ids(c, st, tgt));
    TRY(reset_finished(c, st, n));
    TRY(launch_step(c, st, d_logits, force));
    if (logits_host) {
        CK(cudaMemcpyAsync(logits_host, d_logits, (size_t)4 * n * g.V, cudaMemcpyDeviceToHost, c->stream));
    }
    int steps = 2;
    const int max_steps = std::min(max_new + 1, m);
    if (capture && !st->exec && steps < max_steps) {
        cudaGraph_t graph = nullptr;
        CK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
        mgb_status cs = launch_step(c, st, nullptr, force);
        cudaError_t ee = cudaStreamEndCapture(c->stream, &graph);
        if (cs != MGB_OK) {
            if (graph) cudaGraphDestroy(graph);
            return cs;
        }
        if (ee != cudaSuccess) return cuda_err(ee, "cudaStreamEndCapture");
        cudaError_t ie = cudaGraphInstantiate(&st->exec, graph, 0);
        size_t nodes = 0;
        cudaGraphGetNodes(graph, nullptr, &nodes);
        cudaGraphDestroy(graph);
        if (ie != cudaSuccess) {
            st->exec = nullptr;
            return cuda_err(ie, "cudaGraphInstantiate");
        }
        st->graph_nodes = nodes;
        c->launches -= nodes;  // captured launches did not run
        CK(cudaGraphUpload(st->exec, c->stream));
    }
    while (steps < max_steps) {
        if (!force && steps % sync_every == 0) {
            std::vector<uint8_t> fin(st->b);
            CK(cudaMemcpyAsync(fin.data(), st->finished, st->b, cudaMemcpyDeviceToHost, c->stream));
            CK(cudaStreamSynchronize(c->stream));
            if (std::all_of(fin.begin(), fin.end(), [](uint8_t v) { return v != 0; })) break;
        }
        if (st->exec) {
            CK(cudaGraphLaunch(st->exec, c->stream));
            c->launches += st->graph_nodes;
        } else {
            TRY(launch_step(c, st, d_logits, force));
            if (logits_host)
                CK(cudaMemcpyAsync(logits_host + (size_t)(steps - 1) * n * g.V, d_logits, (size_t)4 * n * g.V,
                                   cudaMemcpyDeviceToHost, c->stream));
        }
        ++steps;
    }
    std::vector<uint32_t> out((size_t)st->b * st->m);
    uint32_t derr = 0;
    CK(cudaMemcpyAsync(out.data(), st->out, 4 * out.size(), cudaMemcpyDeviceToHost, c->stream));
    CK(cudaMemcpyAsync(&derr, c->d_err, 4, cudaMemcpyDeviceToHost, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    if (derr) {
        cudaMemsetAsync(c->d_err, 0, 4, c->stream);
        return set_err(MGB_ERR_CUDA, "a device-side wait ran out of time (flags %u)", derr);
    }
    for (int r = 0; r < n; ++r) {
        uint32_t len = 0;
        bool seen = false;
        for (int t = 0; t < max_new; ++t) {
            const uint32_t tok = t < steps - 1 ? out[(size_t)r * st->m + 1 + t] : (uint32_t)g.pad;
            out_ids[(size_t)r * max_new + t] = tok;
            if (!seen && t < steps - 1 && tok != (uint32_t)g.eos) ++len;
            else seen = true;
        }
        if (out_lens) out_lens[r] = len;
    }
    return MGB_OK;
}

// ---------------------------------------------------------------------------
// C ABI

extern "C" {

void mgb_default_options(mgb_options *o) {
    o->use_graphs = 1;
    o->graph_cache_bytes = (uint64_t)8 << 30;
    o->fail_alloc_after = -1;
}

const char *mgb_last_error(void) { return g_err.c_str(); }

mgb_status mgb_open(const char *path, int device, const mgb_options *opts, mgb_ctx **out) {
    if (!path || !out) return set_err(MGB_ERR_INVALID, "null argument");
    *out = nullptr;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0) return set_err(MGB_ERR_CUDA, "no CUDA device available (%s)", cudaGetErrorString(e));
    if (device < 0 || device >= n) return set_err(MGB_ERR_INVALID, "device %d out of range (%d devices)", device, n);
    CK(cudaSetDevice(device));
    auto c = std::make_unique<mgb_ctx>();
    c->device = device;
    if (opts) c->opts = *opts;
    else mgb_default_options(&c->opts);
    CK(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
    if (const char *v = getenv("MGB_TC_MIN_NT")) c->tc_min_nt = atoi(v);
    if (const char *v = getenv("MGB_TC_SPLIT")) c->tc_split = atoi(v) != 0;
    if (const char *v = getenv("MGB_TC_SPLIT_STAGES")) c->tc_split_stages = std::max(1, atoi(v));
    if (const char *v = getenv("MGB_TC_SPLIT_MAX")) c->tc_split_max = std::max(1, atoi(v));
    if (const char *v = getenv("MGB_STEP_KERNEL")) c->step_kernel = atoi(v) != 0;
    if (const char *v = getenv("MGB_STEP_TRACE")) c->step_trace = v;
    if (const char *v = getenv("MGB_TEST_WAIT_NS")) c->test_wait_ns = std::max<uint64_t>(1000, strtoull(v, nullptr, 10));
    if (const char *v = getenv("MGB_TEST_WITHHOLD_CHUNK")) c->test_withhold_chunk = atoi(v);
    if (const char *v = getenv("MGB_TEST_WITHHOLD_TOPK")) c->test_withhold_topk = atoi(v);
    if (const char *v = getenv("MGB_TEST_WITHHOLD_STEP")) c->test_withhold_step = atoi(v);
    if (const char *v = getenv("MGB_FFN_Q8")) c->ffn_q8 = atoi(v) != 0;
    if (const char *v = getenv("MGB_SMALL_CLUSTER")) {
        const int k = atoi(v);
        c->small_cluster = k == 2 || k == 4 || k == 8 ? k : 1;
    }
    cudaDeviceGetAttribute(&c->sms, cudaDevAttrMultiProcessorCount, device);
    if (c->sms <= 0) c->sms = 148;
    {
        int optin = 0;
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
        if (optin > 8192) c->smem_optin = (size_t)optin - 4096;  // room for the kernel's static shared memory
    }
    mgb_status s = load_model(c.get(), path);
    if (s != MGB_OK) {
        if (c->arena) cudaFree(c->arena);
        cudaStreamDestroy(c->stream);
        return s;
    }
    {
        void *p = nullptr;
        mgb_status es = c->dalloc(&p, 4);
        if (es != MGB_OK) {
            cudaFree(c->arena);
            cudaStreamDestroy(c->stream);
            return es;
        }
        c->d_err = (uint32_t *)p;
        CK(cudaMemset(c->d_err, 0, 4));
    }
    c->inject_armed = true;
    count_context(device, 1);
    *out = c.release();
    return MGB_OK;
}

void mgb_close(mgb_ctx *c) {
    if (!c) return;
    cudaSetDevice(c->device);
    for (mgb_batch *B : c->batches) B->owner = nullptr;  // they free their own buffers later
    clear_cache(c);
    if (c->arena) cudaFree(c->arena);
    if (c->d_err) cudaFree(c->d_err);
    cudaStreamDestroy(c->stream);
    count_context(c->device, -1);
    delete c;
}

mgb_status mgb_model_info_get(const mgb_ctx *c, mgb_model_info *o) {
    if (!c || !o) return set_err(MGB_ERR_INVALID, "null argument");
    const Config &g = c->cfg;
    o->vocab_size = g.V;
    o->d_model = g.d;
    o->encoder_layers = g.enc_layers;
    o->decoder_layers = g.dec_layers;
    o->encoder_heads = g.enc_heads;
    o->decoder_heads = g.dec_heads;
    o->encoder_ffn = g.enc_ffn;
    o->decoder_ffn = g.dec_ffn;
    o->max_position_embeddings = g.max_pos;
    o->max_length = g.max_length;
    o->pad_token_id = g.pad;
    o->eos_token_id = g.eos;
    o->decoder_start_token_id = g.start;
    o->bos_token_id = g.bos;
    o->scale_embedding = g.scale_embedding;
    o->weight_bytes = c->weight_bytes;
    o->decoder_step_bytes = c->step_bytes;
    o->lm_head_bytes = c->embed.bytes;
    return MGB_OK;
}

mgb_status mgb_encode(mgb_ctx *c, const uint32_t *ids, const uint32_t *lens, uint32_t b, uint32_t s, mgb_batch **out) {
    if (!c || !ids || !lens || !out) return set_err(MGB_ERR_INVALID, "null argument");
    *out = nullptr;
    if (b == 0 || s == 0) return set_err(MGB_ERR_INVALID, "empty batch");
    if ((int)s > c->cfg.max_pos - 2) return set_err(MGB_ERR_INVALID, "source length %u > %d", s, c->cfg.max_pos - 2);
    for (uint32_t i = 0; i < b; ++i) {
        if (lens[i] < 1 || lens[i] > s) return set_err(MGB_ERR_INVALID, "lens[%u] = %u outside [1, %u]", i, lens[i], s);
        for (uint32_t j = 0; j < lens[i]; ++j)
            if (ids[(size_t)i * s + j] >= (uint32_t)c->cfg.V)
                return set_err(MGB_ERR_INVALID, "token id %u >= vocab %d", ids[(size_t)i * s + j], c->cfg.V);
    }
    CK(cudaSetDevice(c->device));
    // the reference pads a batch to its longest sentence (pad_batch,
    // model.rs:480-500): repack a wider stride
    uint32_t smax = 0;
    for (uint32_t i = 0; i < b; ++i) smax = std::max(smax, lens[i]);
    if (smax == s) return encode(c, ids, lens, (int)b, (int)s, out);
    std::vector<uint32_t> packed((size_t)b * smax);
    for (uint32_t i = 0; i < b; ++i) memcpy(&packed[(size_t)i * smax], ids + (size_t)i * s, 4 * (size_t)smax);
    return encode(c, packed.data(), lens, (int)b, (int)smax, out);
}

void mgb_batch_free(mgb_batch *B) {
    if (!B) return;
    if (B->owner) {
        cudaSetDevice(B->owner->device);
        B->owner->batches.erase(B);
        batch_release(B->owner, B);
    } else {  // its context was closed first
        cudaFree(B->buf);
    }
    delete B;
}

mgb_status mgb_batch_cross(mgb_ctx *c, const mgb_batch *B, uint32_t layer, int which, uint16_t *out) {
    if (!c || !B || !out || layer >= (uint32_t)c->cfg.dec_layers) return set_err(MGB_ERR_INVALID, "bad argument");
    const size_t per = (size_t)B->b * c->cfg.d * B->s;
    std::vector<float> f(per);
    CK(cudaMemcpy(f.data(), B->cross + per * (2 * layer + which), per * 4, cudaMemcpyDeviceToHost));
    for (size_t i = 0; i < per; ++i) out[i] = __half_as_ushort(__float2half_rn(f[i]));
    return MGB_OK;
}

static mgb_status check_greedy(mgb_ctx *c, const mgb_batch *B, uint32_t tgt, uint32_t max_new) {
    if (!c || !B) return set_err(MGB_ERR_INVALID, "null argument");
    if (B->owner != c) return set_err(MGB_ERR_INVALID, "batch belongs to another context");
    if (tgt >= (uint32_t)c->cfg.V) return set_err(MGB_ERR_INVALID, "target language id %u >= vocab", tgt);
    if (max_new < 1 || (int)max_new > c->cfg.max_pos - 2)
        return set_err(MGB_ERR_INVALID, "max_new %u outside [1, %d]", max_new, c->cfg.max_pos - 2);
    return MGB_OK;
}

static mgb_status greedy_api(mgb_ctx *c, const mgb_batch *B, uint32_t tgt, uint32_t max_new, uint32_t sync_every,
                             int force, uint32_t *out_ids, uint32_t *out_lens, int sl) {
    TRY(check_greedy(c, B, tgt, max_new));
    if (!out_ids) return set_err(MGB_ERR_INVALID, "null out_ids");
    CK(cudaSetDevice(c->device));
    mgb_status s = run_greedy(c, B, tgt, (int)max_new, std::max(1u, sync_every), force, out_ids, out_lens, nullptr, sl);
    if (s == MGB_OK) return s;
    if (s == MGB_ERR_OOM && c->capture && c->opts.use_graphs) {
        // graph.rs:214-222: drop graphs for good and retry eagerly
        std::string why = g_err;
        c->capture = false;
        clear_cache(c);
        s = run_greedy(c, B, tgt, (int)max_new, std::max(1u, sync_every), force, out_ids, out_lens, nullptr, sl);
        if (s != MGB_OK) g_err = why + "; retry without graphs: " + g_err;
    }
    return s;
}

mgb_status mgb_greedy(mgb_ctx *c, const mgb_batch *B, uint32_t tgt, uint32_t max_new, uint32_t sync_every, int force,
                      uint32_t *out_ids, uint32_t *out_lens) {
    return greedy_api(c, B, tgt, max_new, sync_every, force, out_ids, out_lens, -1);
}

int mgb_shortlist_find(const mgb_ctx *c, const char *code) {
    if (!c || !code) return -1;
    for (size_t i = 0; i < c->shortlists.size(); ++i)
        if (c->shortlists[i].code == code) return (int)i;
    return -1;
}

mgb_status mgb_greedy_shortlist(mgb_ctx *c, const mgb_batch *B, uint32_t tgt, int shortlist, uint32_t max_new,
                                uint32_t sync_every, int force, uint32_t *out_ids, uint32_t *out_lens) {
    if (!c) return set_err(MGB_ERR_INVALID, "null argument");
    if (shortlist < 0 || shortlist >= (int)c->shortlists.size())
        return set_err(MGB_ERR_INVALID, "no shortlist %d", shortlist);
    // the forced start tokens must be in the shortlist (translator.rs:186-192)
    const std::vector<uint32_t> &ids = c->shortlists[shortlist].ids;
    for (uint32_t t : {(uint32_t)c->cfg.start, tgt})
        if (!std::binary_search(ids.begin(), ids.end(), t))
            return set_err(MGB_ERR_INVALID, "token %u missing from shortlist %s", t,
                           c->shortlists[shortlist].code.c_str());
    return greedy_api(c, B, tgt, max_new, sync_every, force, out_ids, out_lens, shortlist);
}

mgb_status mgb_beam(mgb_ctx *c, const mgb_batch *B, uint32_t tgt, uint32_t k, float length_penalty, uint32_t max_new,
                    uint32_t *out_ids, uint32_t *out_lens) {
    TRY(check_greedy(c, B, tgt, max_new));
    if (!out_ids) return set_err(MGB_ERR_INVALID, "null out_ids");
    if (k < 1 || k > 8) return set_err(MGB_ERR_INVALID, "beam width %u outside 1..8", k);
    if ((uint64_t)B->b * k > 64) return set_err(MGB_ERR_INVALID, "batch x beam = %llu rows exceeds 64",
                                                (unsigned long long)B->b * k);
    CK(cudaSetDevice(c->device));
    return run_beam(c, B, tgt, (int)k, length_penalty, (int)max_new, out_ids, out_lens);
}

mgb_status mgb_log_softmax_topk(mgb_ctx *c, const float *logits, uint32_t rows, uint32_t vocab, uint32_t k,
                                float *vals, uint32_t *idx) {
    if (!c || !logits || !vals || !idx) return set_err(MGB_ERR_INVALID, "null argument");
    if (rows == 0 || vocab == 0) return set_err(MGB_ERR_INVALID, "empty input");
    if (k < 1 || k > 8) return set_err(MGB_ERR_INVALID, "k = %u outside 1..8", k);
    if ((uint64_t)rows * vocab > (1ull << 31)) return set_err(MGB_ERR_INVALID, "rows x vocab exceeds 2^31");
    CK(cudaSetDevice(c->device));
    const size_t n = (size_t)rows * vocab;
    void *d_x = nullptr, *d_v = nullptr, *d_i = nullptr;
    mgb_status s = c->dalloc(&d_x, 4 * n + 16);
    if (s == MGB_OK) s = c->dalloc(&d_v, (size_t)4 * rows * k);
    if (s == MGB_OK) s = c->dalloc(&d_i, (size_t)4 * rows * k);
    uint32_t derr = 0;
    if (s == MGB_OK) {
        cudaMemcpyAsync(d_x, logits, 4 * n, cudaMemcpyHostToDevice, c->stream);
        s = beam_topk(c, (const float *)d_x, (int)rows, (int)vocab, (int)k, (float *)d_v, (uint32_t *)d_i);
    }
    if (s == MGB_OK) {
        cudaMemcpyAsync(vals, d_v, (size_t)4 * rows * k, cudaMemcpyDeviceToHost, c->stream);
        cudaMemcpyAsync(idx, d_i, (size_t)4 * rows * k, cudaMemcpyDeviceToHost, c->stream);
        cudaMemcpyAsync(&derr, c->d_err, 4, cudaMemcpyDeviceToHost, c->stream);
        if (cudaStreamSynchronize(c->stream) != cudaSuccess) s = cuda_err(cudaGetLastError(), "top-k");
    }
    if (s == MGB_OK && derr) {
        cudaMemsetAsync(c->d_err, 0, 4, c->stream);
        s = set_err(MGB_ERR_CUDA, "a device-side wait ran out of time (flags %u)", derr);
    }
    for (void *p : {d_x, d_v, d_i})
        if (p) cudaFree(p);
    return s;
}

mgb_status mgb_greedy_logits(mgb_ctx *c, const mgb_batch *B, uint32_t tgt, uint32_t max_new, int force,
                             uint32_t *out_ids, float *logits) {
    TRY(check_greedy(c, B, tgt, max_new));
    if (!out_ids) return set_err(MGB_ERR_INVALID, "null out_ids");
    CK(cudaSetDevice(c->device));
    std::vector<float> dummy;
    float *lg = logits;
    if (!lg) {
        dummy.resize((size_t)max_new * B->b * c->cfg.V);
        lg = dummy.data();
    }
    return run_greedy(c, B, tgt, (int)max_new, 1 << 30, force, out_ids, nullptr, lg);
}

mgb_status mgb_clear_cache(mgb_ctx *c) {
    if (!c) return set_err(MGB_ERR_INVALID, "null argument");
    CK(cudaSetDevice(c->device));
    clear_cache(c);
    return MGB_OK;
}

void *mgb_cuda_stream(mgb_ctx *c) { return c ? (void *)c->stream : nullptr; }

uint64_t mgb_kernel_launches(const mgb_ctx *c) { return c ? c->launches : 0; }

mgb_status mgb_profile_step(mgb_ctx *c, const mgb_batch *B, uint32_t tgt, uint32_t iters, float *lm_head_ms,
                            float *step_ms) {
    TRY(check_greedy(c, B, tgt, iters + 1));
    CK(cudaSetDevice(c->device));
    StaticState *st = nullptr;
    TRY(acquire_state(c, B, (int)iters + 1, true, &st));
    TRY(set_ids(c, st, tgt));
    cudaEvent_t ev[4];
    for (auto &e : ev) CK(cudaEventCreate(&e));
    double lm = 0.0, step = 0.0;
    mgb_status s = MGB_OK;
    for (uint32_t i = 0; i < iters && s == MGB_OK; ++i) {
        cudaEventRecord(ev[0], c->stream);
        s = launch_step(c, st, nullptr, 1, ev[1], ev[2]);
        cudaEventRecord(ev[3], c->stream);
        if (cudaEventSynchronize(ev[3]) != cudaSuccess) s = cuda_err(cudaGetLastError(), "profile");
        float a = 0.f, b = 0.f;
        cudaEventElapsedTime(&a, ev[1], ev[2]);
        cudaEventElapsedTime(&b, ev[0], ev[3]);
        lm += a;
        step += b;
    }
    for (auto &e : ev) cudaEventDestroy(e);
    if (lm_head_ms) *lm_head_ms = (float)(lm / std::max(1u, iters));
    if (step_ms) *step_ms = (float)(step / std::max(1u, iters));
    return s;
}

}  // extern "C"
