// C ABI of the B200 MoE FFN library: the reference engine's MoE entry points (same names,
// signatures and argument meaning) plus draco_b200_* extensions, over the kernels of
// route.cu / gemv.cu / q8k.cu.
//
// Host side: one context per CUDA device (stream, weight registry, workspace arena), a
// process-wide mutex (the reference's callers are single-threaded too), thread-local error
// text.  Weights arrive as the caller's addresses; host ranges are copied to device memory
// once, on first use, and found again by address on later calls.
#include "../../include/draco_moe_b200.h"
#include "kernels.cuh"
#include "tc_gemm.cuh"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <initializer_list>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

using namespace draco;

extern "C" {
double m6_prof_t[24];
long m6_prof_n[24];
}

namespace {

thread_local std::string g_err;
std::mutex g_mu;
int g_act_mode = 0;
int g_moe_chunk = 64;
// grouped GEMM path: 0 automatic, 1 CUDA cores, 2 tensor cores (where supported)
int g_gemm_path = -1;
int gemm_path() {
    if (g_gemm_path < 0) {
        const char* v = getenv("DRACO_B200_GEMM");
        g_gemm_path = v ? atoi(v) : 0;
    }
    return g_gemm_path;
}
int tc_min_assignments() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("DRACO_B200_TC_MIN_P");
        v = e ? atoi(e) : 128;
    }
    return v;
}
long g_launches = 0;          // kernels this library launched (all devices)

// Optional per-phase device timing: CUDA events recorded around each phase on the launching
// stream, resolved when read.
enum Phase { kRoute = 0, kDispatch, kGateUp, kDown, kShared, kCombine, kGather, kFused, kPhases };
bool g_prof = false;
struct PendingEv {
    int phase;
    cudaEvent_t a, b;
};
std::vector<PendingEv> g_pending;
std::vector<cudaEvent_t> g_ev_pool;
double g_phase_ms[kPhases];
long g_phase_n[kPhases];

cudaEvent_t ev_get() {
    if (!g_ev_pool.empty()) {
        cudaEvent_t e = g_ev_pool.back();
        g_ev_pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

struct PhaseScope {
    int phase;
    cudaStream_t s;
    cudaEvent_t a = nullptr;
    PhaseScope(int p, cudaStream_t st) : phase(p), s(st) {
        if (g_prof) {
            a = ev_get();
            cudaEventRecord(a, s);
        }
    }
    // nothing ran in this scope (a launch that did not happen): record nothing
    void drop() {
        if (a) g_ev_pool.push_back(a);
        a = nullptr;
    }
    ~PhaseScope() {
        if (g_prof && a) {
            cudaEvent_t b = ev_get();
            cudaEventRecord(b, s);
            g_pending.push_back(PendingEv{phase, a, b});
        }
    }
};

void resolve_prof() {
    for (auto& p : g_pending) {
        cudaEventSynchronize(p.b);
        float ms = 0.f;
        if (cudaEventElapsedTime(&ms, p.a, p.b) == cudaSuccess) {
            g_phase_ms[p.phase] += ms;
            g_phase_n[p.phase]++;
        }
        g_ev_pool.push_back(p.a);
        g_ev_pool.push_back(p.b);
    }
    g_pending.clear();
}

void set_err(const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
}

bool env_flag(const char* name) {
    const char* v = getenv(name);
    return v && v[0] && strcmp(v, "0") != 0;
}

// Report an error of a `void` entry point: stderr, NaN output, optional abort.
void fail_void(const char* fn, float* out, size_t n) {
    fprintf(stderr, "[draco_moe_b200] %s: %s\n", fn, g_err.c_str());
    if (env_flag("DRACO_B200_STRICT")) abort();
    if (out)
        for (size_t i = 0; i < n; i++) out[i] = NAN;
}

#define CK(call)                                                                         \
    do {                                                                                 \
        cudaError_t e_ = (call);                                                         \
        if (e_ != cudaSuccess) {                                                         \
            set_err("%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, __LINE__); \
            return -3;                                                                   \
        }                                                                                \
    } while (0)

double now_s() {
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// A device copy of one host range.  `subs` records, for every exact (address, length) range a
// caller has asked for inside it, the content signature of those host bytes when they were
// last copied.  Only the bytes of the range named in the current call are ever read: a range
// whose signature changed (the caller freed its buffer and a new one took the address, or
// rewrote it) is copied again into the same device bytes, so device addresses stay stable.
struct Region {
    uintptr_t host;
    size_t bytes;
    void* dev;
    std::map<std::pair<uintptr_t, size_t>, uint64_t> subs;
    // Q6_K copy padded to 224-byte superblocks: n_mats matrices of rows x nb superblocks, host_per
    // bytes apart on the host side, dev_per apart on the device.  rows == 0: plain byte copy.
    int rows = 0, nb = 0, n_mats = 0;
    size_t host_per = 0, dev_per = 0;
    bool from_device = false;   // copied from caller device memory (no host bytes to re-check)
};

// After an in-place copy of host range [h, h + bytes) into a region, the device bytes of every
// other recorded sub-range that overlaps it are no longer that sub-range's contents: forget
// them, so their next lookup copies again instead of trusting a matching signature.
void forget_overlaps(Region& r, uintptr_t h, size_t bytes) {
    for (auto it = r.subs.begin(); it != r.subs.end();) {
        const uintptr_t a = it->first.first;
        const size_t n = it->first.second;
        if (a < h + bytes && h < a + n && !(a == h && n == bytes)) it = r.subs.erase(it);
        else ++it;
    }
}

// Signature of a host range from 16 sampled 8-byte words (first, last, evenly between).
uint64_t host_sig(const void* p, size_t bytes) {
    const uint8_t* b = (const uint8_t*)p;
    uint64_t h = 1469598103934665603ull ^ (uint64_t)bytes;
    const int S = 16;
    for (int i = 0; i < S; i++) {
        const size_t off = bytes <= 8 ? 0 : (size_t)((unsigned __int128)(bytes - 8) * i / (S - 1));
        uint64_t w = 0;
        memcpy(&w, b + off, bytes < 8 ? bytes : 8);
        h = (h ^ w) * 1099511628211ull;
    }
    return h;
}

// one weight-matrix request: host base, format, rows, row length, matrices, host stride
struct MatKey {
    uintptr_t host;
    int code, rows, n_in, n_mats;
    size_t host_per;
    const uint8_t* dev;    // what it resolved to
    size_t dev_per;
};

struct Table {
    std::vector<uint64_t> ptrs;
    std::vector<int> codes;
    std::vector<MatKey> mats;        // the caller ranges the table points into
    int n = 0;
    const uint8_t** d_w = nullptr;   // device array of 3n device addresses
    int cg = 0, cu = 0, cd = 0;
    int q6s = kQ6Padded;             // Q6_K superblock stride of the device copies
    bool stacked = false;            // each matrix kind is base + e * dev_per[k]
    const uint8_t* base[3] = {nullptr, nullptr, nullptr};
    size_t dev_per[3] = {0, 0, 0};
    int inter = 0, n_in = 0, n_out = 0;
    void* tc = nullptr;              // tensor-core path state (tensor maps), owned by tc_gemm.cu
    bool aligned16 = false;          // every matrix starts on a 16-byte boundary (bulk copies)
};

struct Ctx {
    int dev = -1;
    cudaStream_t stream = nullptr;
    std::map<uintptr_t, Region> regions;
    size_t reg_bytes = 0;
    std::map<std::tuple<uintptr_t, int, int, int, int>, Table> tables;
    char* ws = nullptr;
    size_t ws_cap = 0;
    int* d_consts = nullptr;     // [0] = 0, [1] = 1, [2..3] = {0, T} (dense single-expert lists)
    unsigned long gen = 0;       // bumped whenever cached tables are dropped
    // the workspace is shared by all calls: each call's stream waits for the previous call's
    // last use of it (recorded on its stream) before its first use
    cudaEvent_t ws_event = nullptr;
    bool ws_event_set = false;
    cudaEvent_t legacy_event = nullptr;   // orders the library stream after the legacy default stream
    cudaStream_t aux_stream = nullptr;    // second copy stream: large host->device copies run as two halves
    cudaEvent_t aux_fork = nullptr, aux_join = nullptr;
    int* h_status = nullptr;              // page-locked [2]: status words read back by graph-replayed host calls
    // set once a call was captured into an application's CUDA graph: that graph keeps the
    // workspace addresses, so a workspace that is outgrown is retired instead of freed
    bool ws_captured = false;
    std::vector<char*> ws_retired;
    // captured launch sequences of asynchronous device-pointer layer calls
    struct Graph {
        std::vector<uint64_t> key;
        cudaGraphExec_t exec = nullptr;
        long launches = 0;
        unsigned long last_use = 0;
    };
    std::vector<Graph> graphs;
    unsigned long graph_clock = 0;
};

Ctx* g_ctx[64];

// Host -> device copy that is complete on return.  cudaMemcpy from pageable memory may return
// once the data is staged, before the DMA lands, and the library's kernels run on a non-blocking
// stream that does not wait for the legacy stream the copy runs on.
cudaError_t upload_sync(void* d, const void* h, size_t n) {
    cudaError_t e = cudaMemcpy(d, h, n, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    return e;
}

bool is_device_ptr(const void* p) {
    if (!p) return false;
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

Ctx* get_ctx() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        set_err("no CUDA device available");
        return nullptr;
    }
    if (dev < 0 || dev >= 64) {
        set_err("device index %d out of range", dev);
        return nullptr;
    }
    if (!g_ctx[dev]) {
        Ctx* c = new Ctx();
        c->dev = dev;
        if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess ||
            cudaMalloc(&c->d_consts, 4 * sizeof(int)) != cudaSuccess ||
            cudaEventCreateWithFlags(&c->ws_event, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&c->legacy_event, cudaEventDisableTiming) != cudaSuccess ||
            cudaStreamCreateWithFlags(&c->aux_stream, cudaStreamNonBlocking) != cudaSuccess ||
            cudaEventCreateWithFlags(&c->aux_fork, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&c->aux_join, cudaEventDisableTiming) != cudaSuccess ||
            cudaMallocHost((void**)&c->h_status, 2 * sizeof(int)) != cudaSuccess) {
            set_err("CUDA context set-up failed: %s", cudaGetErrorString(cudaGetLastError()));
            delete c;
            return nullptr;
        }
        const int init[4] = {0, 1, 0, 0};
        upload_sync(c->d_consts, init, sizeof init);
        g_ctx[dev] = c;
    }
    return g_ctx[dev];
}

// Device buffers handed over without a stream may have been written on the legacy default
// stream (a framework's default stream), which the library's non-blocking stream does not wait
// for by itself.
int after_legacy_stream(Ctx* c) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(c->stream, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) {
        cudaGetLastError();
        return 0;
    }
    if (cudaEventRecord(c->legacy_event, cudaStreamLegacy) != cudaSuccess ||
        cudaStreamWaitEvent(c->stream, c->legacy_event, 0) != cudaSuccess) {
        set_err("ordering after the default stream failed: %s", cudaGetErrorString(cudaGetLastError()));
        return -3;
    }
    return 0;
}

bool is_pinned_host(const void* p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeHost;
}

// Host -> device copy of activations on stream s.  From page-locked memory a copy of 1 MiB or
// more goes as two halves on two streams (two copy engines): measured on B200, 4 MiB took
// ~145 us as one copy and ~105 us as two.
int h2d(Ctx* c, void* dst, const void* src, size_t bytes, cudaStream_t s) {
    if (bytes < ((size_t)1 << 20) || !is_pinned_host(src)) {
        CK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, s));
        return 0;
    }
    const size_t half = (bytes / 2) & ~(size_t)4095;
    CK(cudaEventRecord(c->aux_fork, s));
    CK(cudaStreamWaitEvent(c->aux_stream, c->aux_fork, 0));
    CK(cudaMemcpyAsync((char*)dst + half, (const char*)src + half, bytes - half, cudaMemcpyHostToDevice,
                       c->aux_stream));
    CK(cudaEventRecord(c->aux_join, c->aux_stream));
    CK(cudaMemcpyAsync(dst, src, half, cudaMemcpyHostToDevice, s));
    CK(cudaStreamWaitEvent(s, c->aux_join, 0));
    return 0;
}

void free_table(Table& t) {
    cudaFree((void*)t.d_w);
    delete (TcMaps*)t.tc;
    t.tc = nullptr;
}

void drop_graphs(Ctx* c);

void drop_tables(Ctx* c) {
    for (auto& kv : c->tables) free_table(kv.second);
    c->tables.clear();
    c->gen++;
    drop_graphs(c);   // they launch kernels on the dropped tables' device data
}

void drop_region(Ctx* c, std::map<uintptr_t, Region>::iterator it) {
    cudaDeviceSynchronize();
    drop_tables(c);   // tables may point into the range
    cudaFree(it->second.dev);
    c->reg_bytes -= it->second.bytes;
    c->regions.erase(it);
}

// device address of host range [host, host+bytes): existing copy (refreshed if the host
// bytes changed), or a new one.
const uint8_t* dev_range(Ctx* c, const void* host, size_t bytes) {
    if (!host || bytes == 0) {
        set_err("null or empty weight range");
        return nullptr;
    }
    const uintptr_t h = (uintptr_t)host;
    auto it = c->regions.upper_bound(h);
    while (it != c->regions.begin()) {
        --it;
        Region& r = it->second;
        if (r.rows == 0 && r.host <= h && h + bytes <= r.host + r.bytes) {
            const uint64_t sig = host_sig(host, bytes);
            auto sub = r.subs.find(std::make_pair(h, bytes));
            uint8_t* d = (uint8_t*)r.dev + (h - r.host);
            if (sub == r.subs.end() || sub->second != sig) {
                // new or changed contents at a known address: copy them again, in place
                cudaDeviceSynchronize();
                if (upload_sync(d, host, bytes) != cudaSuccess) {
                    set_err("weight refresh failed: %s", cudaGetErrorString(cudaGetLastError()));
                    return nullptr;
                }
                forget_overlaps(r, h, bytes);
                r.subs[std::make_pair(h, bytes)] = sig;
            }
            return d;
        }
        if (r.host + (size_t(1) << 40) < h) break;   // regions are never that large
    }
    if (is_device_ptr(host)) return (const uint8_t*)host;
    auto same = c->regions.find(h);
    if (same != c->regions.end()) drop_region(c, same);   // a longer range now starts here
    void* d = nullptr;
    if (cudaMalloc(&d, bytes) != cudaSuccess) {
        set_err("cudaMalloc of %zu weight bytes failed: %s", bytes, cudaGetErrorString(cudaGetLastError()));
        return nullptr;
    }
    if (upload_sync(d, host, bytes) != cudaSuccess) {
        set_err("weight upload failed: %s", cudaGetErrorString(cudaGetLastError()));
        cudaFree(d);
        return nullptr;
    }
    Region r{h, bytes, d, {}};
    r.subs[std::make_pair(h, bytes)] = host_sig(host, bytes);
    c->regions[h] = std::move(r);
    c->reg_bytes += bytes;
    return (const uint8_t*)d;
}

// Copy n_mats Q6_K matrices (rows x nb superblocks each, src_per bytes apart, host or device
// memory) into dst with 224-byte superblocks.
int upload_q6(void* dst, const void* src, bool src_dev, int n_mats, size_t src_per, int rows, int nb) {
    const size_t mat = (size_t)rows * nb * kQ6File;
    if (src_dev) {
        launch_q6_pad((const uint8_t*)src, src_per, n_mats, rows, nb, (uint8_t*)dst, 0);
        CK(cudaGetLastError());
        CK(cudaDeviceSynchronize());
        return 0;
    }
    uint8_t* tmp = nullptr;
    CK(cudaMalloc((void**)&tmp, mat * n_mats));
    cudaError_t e = cudaMemcpy2D(tmp, mat, src, src_per, mat, n_mats, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) {
        launch_q6_pad(tmp, mat, n_mats, rows, nb, (uint8_t*)dst, 0);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    cudaFree(tmp);
    if (e != cudaSuccess) {
        set_err("Q6_K weight upload failed: %s", cudaGetErrorString(e));
        return -3;
    }
    return 0;
}

// Device copy of n_mats weight matrices of `code` (rows x n_in values each, host_per bytes
// apart) starting at `host`; *dev_per receives the device distance between matrices.  Q6_K
// copies are padded to 224-byte superblocks; other formats are byte copies (dev_range).
const uint8_t* dev_matrix(Ctx* c, const void* host, int code, int rows, int n_in, int n_mats, size_t host_per,
                          size_t* dev_per) {
    const size_t mat = (size_t)rows * row_bytes(code, n_in);
    if (n_mats <= 1) host_per = mat;
    const size_t bytes = host_per * (n_mats - 1) + mat;
    if (code != DRACO_CODE_Q6_K) {
        *dev_per = host_per;
        return dev_range(c, host, bytes);
    }
    const int nb = n_in / 256;
    const uintptr_t h = (uintptr_t)host;
    auto it = c->regions.upper_bound(h);
    while (it != c->regions.begin()) {
        --it;
        Region& r = it->second;
        if (r.rows == rows && r.nb == nb && r.host <= h && h + bytes <= r.host + r.bytes &&
            (h - r.host) % r.host_per == 0 && (n_mats == 1 || host_per == r.host_per)) {
            const size_t m0 = (h - r.host) / r.host_per;
            if (m0 + n_mats <= (size_t)r.n_mats) {
                uint8_t* d = (uint8_t*)r.dev + m0 * r.dev_per;
                if (!r.from_device) {
                    const uint64_t sig = host_sig(host, bytes);
                    auto sub = r.subs.find(std::make_pair(h, bytes));
                    if (sub == r.subs.end() || sub->second != sig) {
                        cudaDeviceSynchronize();
                        if (upload_q6(d, host, false, n_mats, host_per, rows, nb)) return nullptr;
                        forget_overlaps(r, h, bytes);
                        r.subs[std::make_pair(h, bytes)] = sig;
                    }
                }
                *dev_per = r.dev_per;
                return d;
            }
        }
        if (r.host + (size_t(1) << 40) < h) break;
    }
    const bool src_dev = is_device_ptr(host);
    auto same = c->regions.find(h);
    if (same != c->regions.end()) drop_region(c, same);
    const size_t dper = (size_t)rows * nb * kQ6Padded;
    void* d = nullptr;
    if (cudaMalloc(&d, dper * n_mats) != cudaSuccess) {
        set_err("cudaMalloc of %zu weight bytes failed: %s", dper * n_mats, cudaGetErrorString(cudaGetLastError()));
        return nullptr;
    }
    if (upload_q6(d, host, src_dev, n_mats, host_per, rows, nb)) {
        cudaFree(d);
        return nullptr;
    }
    Region r{h, bytes, d, {}};
    r.rows = rows;
    r.nb = nb;
    r.n_mats = n_mats;
    r.host_per = host_per;
    r.dev_per = dper;
    r.from_device = src_dev;
    if (!src_dev) r.subs[std::make_pair(h, bytes)] = host_sig(host, bytes);
    c->regions[h] = std::move(r);
    c->reg_bytes += dper * n_mats;
    *dev_per = dper;
    return (const uint8_t*)d;
}

// A cached table is valid while each of its matrices still resolves to the same device bytes
// (contents are refreshed in place when they changed).
bool table_fresh(Ctx* c, const Table& t) {
    const unsigned long gen0 = c->gen;
    const auto mats = t.mats;   // resolving may drop tables (t included): iterate a copy
    for (const auto& m : mats) {
        size_t dp = 0;
        const uint8_t* d = dev_matrix(c, (const void*)m.host, m.code, m.rows, m.n_in, m.n_mats, m.host_per, &dp);
        if (c->gen != gen0 || d != m.dev) return false;
    }
    return true;
}

// activations/outputs: device pointers are used in place, host ones staged
bool dev_kind(const void* p) { return is_device_ptr(p); }

// Resolve a [3n] (gate, up, down) pointer table to device addresses; cached per table
// address and validated against its current contents on every call.
Table* get_table(Ctx* c, const uint64_t* ptrs, const int* codes, int n, int inter, int n_in, int n_out,
                 uintptr_t key_addr = 0) {
    auto key = std::make_tuple(key_addr ? key_addr : (uintptr_t)ptrs, n, inter, n_in, n_out);
    auto it = c->tables.find(key);
    if (it != c->tables.end()) {
        Table& t = it->second;
        if (memcmp(t.ptrs.data(), ptrs, sizeof(uint64_t) * 3 * n) == 0 &&
            memcmp(t.codes.data(), codes, sizeof(int) * 3 * n) == 0) {
            const unsigned long gen0 = c->gen;
            if (table_fresh(c, t)) return &t;
            if (c->gen != gen0) it = c->tables.find(key);   // tables were dropped meanwhile
        }
        if (it != c->tables.end()) {
            free_table(it->second);
            c->tables.erase(it);
        }
    }
    Table t;
    t.n = n;
    t.ptrs.assign(ptrs, ptrs + 3 * n);
    t.codes.assign(codes, codes + 3 * n);
    t.cg = codes[0];
    t.cu = codes[1];
    t.cd = codes[2];
    for (int e = 0; e < n; e++)
        if (codes[3 * e] != t.cg || codes[3 * e + 1] != t.cu || codes[3 * e + 2] != t.cd) {
            set_err("expert %d has formats (%d,%d,%d) != expert 0 (%d,%d,%d); mixed formats unsupported", e,
                    codes[3 * e], codes[3 * e + 1], codes[3 * e + 2], t.cg, t.cu, t.cd);
            return nullptr;
        }
    for (int k = 0; k < 3; k++)
        if (!code_supported(codes[k])) {
            set_err("unsupported weight format code %d", codes[k]);
            return nullptr;
        }
    if (n_in % block_values(t.cg) || n_in % block_values(t.cu) || inter % block_values(t.cd)) {
        set_err("row lengths (n_in %d, inter %d) not a multiple of the block size", n_in, inter);
        return nullptr;
    }
    if ((t.cg != DRACO_CODE_Q8_0 && n_in % 256) || (t.cd != DRACO_CODE_Q8_0 && inter % 256)) {
        set_err("K-quant rows need multiples of 256 values");
        return nullptr;
    }
    const int kcode[3] = {t.cg, t.cu, t.cd};
    const int krows[3] = {inter, inter, n_out};
    const int kin[3] = {n_in, n_in, inter};
    t.inter = inter;
    t.n_in = n_in;
    t.n_out = n_out;
    t.stacked = n > 1;
    std::vector<uint64_t> dptr(3 * n);
    for (int k = 0; k < 3; k++) {
        // stacked experts base + e*per (the GGUF layout) are copied as one range
        const size_t mat = (size_t)krows[k] * row_bytes(kcode[k], kin[k]);
        bool stacked = n > 1;
        const uint64_t base = ptrs[k];
        const uint64_t per = n > 1 ? ptrs[3 + k] - base : 0;
        if (n > 1 && (ptrs[3 + k] <= base || per < mat)) stacked = false;
        for (int e = 2; stacked && e < n; e++)
            if (ptrs[3 * e + k] != base + per * (uint64_t)e) stacked = false;
        if (stacked) {
            size_t dp = 0;
            const uint8_t* d = dev_matrix(c, (const void*)(uintptr_t)base, kcode[k], krows[k], kin[k], n, per, &dp);
            if (!d) return nullptr;
            t.mats.push_back(MatKey{(uintptr_t)base, kcode[k], krows[k], kin[k], n, per, d, dp});
            t.base[k] = d;
            t.dev_per[k] = dp;
            for (int e = 0; e < n; e++) dptr[3 * e + k] = (uint64_t)(uintptr_t)(d + dp * e);
        } else {
            t.stacked = false;
            size_t dp0 = 0;
            for (int e = 0; e < n; e++) {
                size_t dp = 0;
                const uint8_t* d = dev_matrix(c, (const void*)(uintptr_t)ptrs[3 * e + k], kcode[k], krows[k], kin[k],
                                              1, mat, &dp);
                if (!d) return nullptr;
                t.mats.push_back(MatKey{(uintptr_t)ptrs[3 * e + k], kcode[k], krows[k], kin[k], 1, mat, d, dp});
                dptr[3 * e + k] = (uint64_t)(uintptr_t)d;
                if (e == 0) dp0 = dp;
            }
            if (n == 1) {
                t.base[k] = (const uint8_t*)(uintptr_t)dptr[k];
                t.dev_per[k] = dp0;   // the device copy's size (Q6_K padded)
            }
        }
    }
    t.aligned16 = true;
    for (int e = 0; e < 3 * n; e++) {
        const int code = e % 3 == 0 ? t.cg : e % 3 == 1 ? t.cu : t.cd;
        if (dptr[e] % 2 || (code == DRACO_CODE_Q4_K && dptr[e] % 16)) {
            set_err("weight address 0x%llx misaligned for its format", (unsigned long long)dptr[e]);
            return nullptr;
        }
        if (dptr[e] % 16) t.aligned16 = false;
    }
    // an upload made while building this table may have dropped cached tables; the matrices
    // resolved above must still resolve to the same device bytes
    for (auto& m : t.mats) {
        size_t dp = 0;
        if (dev_matrix(c, (const void*)m.host, m.code, m.rows, m.n_in, m.n_mats, m.host_per, &dp) != m.dev) {
            set_err("weight ranges moved while resolving the expert table");
            return nullptr;
        }
    }
    if (cudaMalloc((void**)&t.d_w, sizeof(uint64_t) * 3 * n) != cudaSuccess ||
        upload_sync((void*)t.d_w, dptr.data(), sizeof(uint64_t) * 3 * n) != cudaSuccess) {
        set_err("pointer table upload failed: %s", cudaGetErrorString(cudaGetLastError()));
        return nullptr;
    }
    // tensor-core path: stacked, densely packed copies of supported formats
    if ((t.stacked || n == 1) && tc_supported(t.cg, t.cu, t.cd, inter, n_in, n_out) &&
        t.dev_per[0] == (size_t)inter * row_bytes(t.cg, n_in, t.q6s) &&
        t.dev_per[1] == (size_t)inter * row_bytes(t.cu, n_in, t.q6s) &&
        t.dev_per[2] == (size_t)n_out * row_bytes(t.cd, inter, t.q6s)) {
        TcMaps* m = new TcMaps();
        if (tc_make_weight_maps(m, t.base[0], t.base[1], t.base[2], n, t.cg, t.cd, inter, n_in, n_out) == 0) t.tc = m;
        else delete m;
    }
    auto res = c->tables.emplace(key, std::move(t));
    return &res.first->second;
}

// workspace arena: carve aligned sub-buffers, growing the arena when needed
struct Carver {
    size_t off = 0;
    template <typename T>
    size_t take(size_t count) {
        const size_t o = off;
        off = align_up(off + sizeof(T) * (count ? count : 1), 256);
        return o;
    }
};

void drop_graphs(Ctx* c) {
    for (auto& g : c->graphs) cudaGraphExecDestroy(g.exec);
    c->graphs.clear();
}

// order stream s after the previous call's use of the workspace / record this call's use
void ws_acquire(Ctx* c, cudaStream_t s) {
    if (c->ws_event_set) cudaStreamWaitEvent(s, c->ws_event, 0);
}
void ws_release(Ctx* c, cudaStream_t s) {
    cudaEventRecord(c->ws_event, s);
    c->ws_event_set = true;
}

int ensure_ws(Ctx* c, size_t bytes) {
    ws_acquire(c, c->stream);
    if (bytes <= c->ws_cap) return 0;
    CK(cudaStreamSynchronize(c->stream));
    if (c->ws_event_set) CK(cudaEventSynchronize(c->ws_event));   // asynchronous calls are done with it
    drop_graphs(c);
    if (c->ws && c->ws_captured) c->ws_retired.push_back(c->ws);
    else if (c->ws) cudaFree(c->ws);
    c->ws = nullptr;
    c->ws_cap = 0;
    const size_t cap = align_up(bytes + bytes / 2, 1 << 20);
    CK(cudaMalloc((void**)&c->ws, cap));
    c->ws_cap = cap;
    return 0;
}

struct LayerArgs {
    Table* tab = nullptr;
    Table* sh = nullptr;         // shared expert (n = 1) or null
    int sh_ff = 0;
    int E = 0, K = 0, inter = 0, n_in = 0, n_out = 0;
    RouterParams rp{};
    const float* d_gi = nullptr; // router weights (device), null when routing is given
    bool no_routed = false;      // shared expert only
    bool x_half = false;         // b.x holds fp16 rows
    float* const* out_blk = nullptr;   // output row blocks (device array of pointers), or null
    int out_block = 0;                 // rows per block
};

// routing supplied by the caller: rows of ld entries, expert ids minus e_base index the layer's
// experts (others are skipped); order == nullptr means no routed experts at all
struct GivenRoute {
    const int* order = nullptr;
    const float* wtop = nullptr;
    int ld = 0;
    int e_base = 0;
    bool x_half = false;   // X holds fp16 rows (device memory)
    float* const* out_blk = nullptr;   // row q of the result goes to out_blk[q / out_block] + (q % out_block) * n_out
    int out_block = 0;
};

struct LayerBufs {
    RouteBufs rb{};
    float *x, *out, *act, *y, *act_sh, *y_sh;
    float* x_ws = nullptr;          // the workspace's own activation rows
    int8_t* xq;
    float* xd;
    int16_t* xbs;
    __half *xs_h, *act_h;          // tensor-core path operands
    int4 *items_gu, *items_dn;
    int *n_items, *tc_err;
    int* item_tiles = nullptr;     // dispatch scratch for the item lists
    int4 *items_sh_gu = nullptr, *items_sh_dn = nullptr;   // shared expert on the tensor-core path
    int* n_items_sh = nullptr;
    int* fd_ctl = nullptr;         // fused decode: 2 grid barrier words, routing status, GEMV status
    bool use_tc = false, sh_tc = false;
};

// the fused single-launch decode layer (DRACO_B200_FUSED_DECODE=0 or draco_b200_set_fused_decode
// turn it off); g_fd_extra: test hook, grid barrier arrivals the fused kernel waits for beyond
// its own blocks (a block that never arrives)
// graph replay of synchronous calls on page-locked host buffers (DRACO_B200_HOST_GRAPH=0: off)
bool host_graph_enabled() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("DRACO_B200_HOST_GRAPH");
        v = e ? (atoi(e) != 0) : 1;
    }
    return v != 0;
}
int g_fused_decode = -1;
int g_fd_extra = 0;
bool fused_decode_enabled() {
    if (g_fused_decode < 0) {
        const char* e = getenv("DRACO_B200_FUSED_DECODE");
        g_fused_decode = e ? (atoi(e) != 0) : 1;
    }
    return g_fused_decode != 0;
}

bool want_tc(const LayerArgs& a, int T) {
    const int mode = gemm_path();
    if (mode == 1 || !a.tab || !a.tab->tc || g_act_mode == 1) return false;
    if (mode == 2) return true;
    return T * a.K >= tc_min_assignments();
}

// extra_bytes > 0: that many more bytes for the caller at *extra_off
int carve_layer(Ctx* c, const LayerArgs& a, int T, LayerBufs& b, size_t extra_bytes = 0, size_t* extra_off = nullptr) {
    const size_t n = (size_t)T * a.K;
    Carver cv;
    const size_t o_x = cv.take<float>((size_t)T * a.n_in), o_out = cv.take<float>((size_t)T * a.n_out);
    const size_t o_lg = cv.take<float>((size_t)T * a.E), o_ord = cv.take<int>(n), o_w = cv.take<float>(n);
    const size_t o_cnt = cv.take<int>(a.E), o_off = cv.take<int>(a.E + 1), o_il = cv.take<int>(n);
    const size_t o_pos = cv.take<int>(n), o_act = cv.take<int>(a.E), o_na = cv.take<int>(1), o_err = cv.take<int>(1);
    const size_t o_cc = cv.take<int>(dispatch_chunk_ints((int)n, a.E));
    const size_t o_a = cv.take<float>(n * a.inter), o_y = cv.take<float>(n * a.n_out);
    const size_t o_ash = cv.take<float>(a.sh ? (size_t)T * a.sh_ff : 0);
    const size_t o_ysh = cv.take<float>(a.sh ? (size_t)T * a.n_out : 0);
    const bool q8 = g_act_mode == 1;
    const size_t o_xq = cv.take<int8_t>(q8 ? (size_t)T * a.n_in : 0);
    const size_t o_xd = cv.take<float>(q8 ? (size_t)T * (a.n_in / 256) : 0);
    const size_t o_xbs = cv.take<int16_t>(q8 ? (size_t)T * (a.n_in / 256) * 16 : 0);
    b.use_tc = want_tc(a, T);
    const int na_max = std::min(a.E, (int)n);
    const size_t o_xs = cv.take<__half>(b.use_tc ? n * a.n_in : 0);
    const size_t o_ah = cv.take<__half>(b.use_tc ? n * a.inter : 0);
    const size_t o_igu = cv.take<int4>(b.use_tc ? tc_items_capacity((int)n, na_max, tc_tiles_gateup(a.inter)) : 0);
    const size_t o_idn = cv.take<int4>(b.use_tc ? tc_items_capacity((int)n, na_max, tc_tiles_down(a.n_out)) : 0);
    const size_t o_ni = cv.take<int>(2), o_terr = cv.take<int>(1);
    const size_t o_tiles = cv.take<int>(b.use_tc ? a.E : 0);
    // shared expert on the tensor-core path: reuses Xs and act_h after the routed GEMMs
    b.sh_tc = b.use_tc && a.sh && a.sh->tc && (size_t)T * a.sh_ff <= n * a.inter;
    const size_t sh_tiles = (size_t)T / 64 + 1;
    const size_t o_sgu = cv.take<int4>(b.sh_tc ? sh_tiles * tc_tiles_gateup(a.sh_ff) : 0);
    const size_t o_sdn = cv.take<int4>(b.sh_tc ? sh_tiles * tc_tiles_down(a.n_out) : 0);
    const size_t o_nsh = cv.take<int>(2);
    const size_t o_fd = cv.take<int>(4);
    if (extra_bytes) *extra_off = cv.take<char>(extra_bytes);
    if (int rc = ensure_ws(c, cv.off)) return rc;
    char* w = c->ws;
    b.items_sh_gu = (int4*)(w + o_sgu);
    b.items_sh_dn = (int4*)(w + o_sdn);
    b.n_items_sh = (int*)(w + o_nsh);
    b.fd_ctl = (int*)(w + o_fd);
    b.xs_h = (__half*)(w + o_xs);
    b.act_h = (__half*)(w + o_ah);
    b.items_gu = (int4*)(w + o_igu);
    b.items_dn = (int4*)(w + o_idn);
    b.n_items = (int*)(w + o_ni);
    b.tc_err = (int*)(w + o_terr);
    b.item_tiles = (int*)(w + o_tiles);
    b.x = (float*)(w + o_x);
    b.x_ws = b.x;
    b.out = (float*)(w + o_out);
    b.rb.logits = (float*)(w + o_lg);
    b.rb.order = (int*)(w + o_ord);
    b.rb.wtop = (float*)(w + o_w);
    b.rb.counts = (int*)(w + o_cnt);
    b.rb.off = (int*)(w + o_off);
    b.rb.ilist = (int*)(w + o_il);
    b.rb.pos_of = (int*)(w + o_pos);
    b.rb.active = (int*)(w + o_act);
    b.rb.n_active = (int*)(w + o_na);
    b.rb.err = (int*)(w + o_err);
    b.rb.chunk_counts = (int*)(w + o_cc);
    b.act = (float*)(w + o_a);
    b.y = (float*)(w + o_y);
    b.act_sh = (float*)(w + o_ash);
    b.y_sh = (float*)(w + o_ysh);
    b.xq = (int8_t*)(w + o_xq);
    b.xd = (float*)(w + o_xd);
    b.xbs = (int16_t*)(w + o_xbs);
    return 0;
}

// dense one-expert FFN over T token rows: act = silu(G x) * (U x), y = D act
int dense_ffn(Ctx* c, Table* t, int T, const float* x, int ff, int n_in, int n_out, float* act, float* y,
              int* status, cudaStream_t s) {
    launch_set_pair(c->d_consts + 2, 0, T, s);   // the one expert's token list [0, T)
    ExpertTable et{t->d_w};
    {
        PhaseScope ps(kShared, s);
        if (status && t->aligned16 && dec_supported(t->cg, t->cu, t->cd, ff, n_in, n_out, t->q6s)) {
            int rc = launch_dec_gateup(et, t->cg, t->cu, c->d_consts, c->d_consts + 1, 1, c->d_consts + 2, nullptr, 1,
                                       x, ff, n_in, act, t->q6s, status, s);
            if (rc == 0)
                rc = launch_dec_down(et, t->cd, c->d_consts, c->d_consts + 1, 1, c->d_consts + 2, act, ff, n_out, y,
                                     t->q6s, status, s);
            if (rc) {
                set_err("shared-expert GEMV launch failed (%d)", rc);
                return -3;
            }
        } else {
            launch_gateup_codes(et, t->cg, t->cu, c->d_consts, c->d_consts + 1, 1, c->d_consts + 2, nullptr, 1, x,
                                ff, n_in, act, s, t->q6s);
            launch_down_code(et, t->cd, c->d_consts, c->d_consts + 1, 1, c->d_consts + 2, act, ff, n_out, y, s,
                             t->q6s);
        }
    }
    g_launches += 3;
    CK(cudaGetLastError());
    return 0;
}

// Routed experts (+ shared) on device buffers.  Routing is computed when a.d_gi is set,
// otherwise b.rb.order / b.rb.wtop already hold it.
int run_layer(Ctx* c, const LayerArgs& a, int T, LayerBufs& b, cudaStream_t s) {
    RouteBufs& rb = b.rb;
    bool xh = a.x_half;
    if (xh && (!b.use_tc || (a.sh && !b.sh_tc))) {
        // a CUDA-core path reads these rows: widen the fp16 rows to fp32 first
        launch_half_to_float(reinterpret_cast<const __half*>(b.x), b.x_ws, (size_t)T * a.n_in, s);
        g_launches += 1;
        b.x = b.x_ws;
        xh = false;
    }
    // decode batches: the whole layer (routing, experts, combine, shared expert) in one launch
    const bool sh_ok = !a.sh || (a.sh->aligned16 && a.sh->cg == a.tab->cg && a.sh->cu == a.tab->cu &&
                                 a.sh->cd == a.tab->cd && a.sh->q6s == a.tab->q6s &&
                                 dec_supported(a.sh->cg, a.sh->cu, a.sh->cd, a.sh_ff, a.n_in, a.n_out, a.sh->q6s));
    if (!a.no_routed && !xh && !b.use_tc && !a.out_blk && g_act_mode == 0 && fused_decode_enabled() && T <= 8 &&
        T * a.K <= 64 &&
        a.tab->aligned16 && a.tab->cg == a.tab->cu && sh_ok &&
        dec_supported(a.tab->cg, a.tab->cu, a.tab->cd, a.inter, a.n_in, a.n_out, a.tab->q6s)) {
        FusedDecodeArgs f{};
        f.tab = ExpertTable{a.tab->d_w};
        if (a.sh) {
            f.sh_g = a.sh->base[0];
            f.sh_u = a.sh->base[1];
            f.sh_d = a.sh->base[2];
            f.sh_ff = a.sh_ff;
        }
        f.W = a.d_gi;
        f.rp = a.rp;   // scoring etc. (used only when the router runs here)
        f.rp.n_exp = a.E;
        f.rp.n_used = a.K;
        f.rp.n_in = a.n_in;
        f.X = b.x;
        f.T = T;
        f.F = a.inter;
        f.n_out = a.n_out;
        f.out = b.out;
        f.order = rb.order;
        f.wtop = rb.wtop;
        f.logits = rb.logits;
        f.act = b.act;
        f.act_sh = b.act_sh;
        f.bar = reinterpret_cast<unsigned*>(b.fd_ctl);
        f.route_err = b.fd_ctl + 2;
        f.status = b.fd_ctl + 3;
        f.q6s = a.tab->q6s;
        f.bar_extra = g_fd_extra;
        static unsigned long long* fd_stamps = nullptr;   // DRACO_B200_FD_STATS=1: phase timestamps
        if (!fd_stamps && env_flag("DRACO_B200_FD_STATS")) {
            // device memory (a managed buffer would migrate to the host and back between calls)
            cudaMalloc(&fd_stamps, sizeof(unsigned long long) * 128 * 4096);
            cudaMemset(fd_stamps, 0, sizeof(unsigned long long) * 128 * 4096);
        }
        f.stamps = fd_stamps;
        CK(cudaMemsetAsync(b.fd_ctl, 0, 4 * sizeof(int), s));
        int rc;
        {
            PhaseScope ps(kFused, s);
            rc = launch_fused_decode(f, a.tab->cg, a.tab->cu, a.tab->cd, s);
            if (rc != 0) ps.drop();
        }
        if (rc == 0) {
            rb.err = f.route_err;   // the status words the synchronous calls read back
            b.tc_err = f.status;
            g_launches += 1;
            if (fd_stamps) {
                // per phase: median and max over the blocks of the time since the block started
                cudaStreamSynchronize(s);
                std::vector<unsigned long long> hs((size_t)128 * 4096);
                cudaMemcpy(hs.data(), fd_stamps, sizeof(unsigned long long) * hs.size(), cudaMemcpyDeviceToHost);
                cudaMemset(fd_stamps, 0, sizeof(unsigned long long) * hs.size());
                const unsigned long long* st = hs.data();
                int G = 0;
                while (G < 4096 && st[(size_t)G * 128] != 0) G++;
                fprintf(stderr, "[fused decode stats] blocks=%d", G);
                static const char* nm[7] = {"start", "A", "bar1", "S", "B", "bar2", "C"};
                for (int i : {1, 2, 66, 64, 65, 3, 4, 5, 6}) {
                    std::vector<double> v;
                    for (int g = 0; g < G; g++)
                        if (st[(size_t)g * 128 + i]) v.push_back((st[(size_t)g * 128 + i] - st[(size_t)g * 128]) * 1e-3);
                    std::sort(v.begin(), v.end());
                    if (!v.empty())
                        fprintf(stderr, " %s=%.1f/%.1fus", i < 7 ? nm[i] : i == 66 ? "S:logits" : i == 64 ? "S:select" : "S:list",
                                v[v.size() / 2], v.back());
                }
                for (int blk : {0, G / 2}) {
                    if (blk >= G) continue;
                    const unsigned long long* sb = st + (size_t)blk * 128;
                    fprintf(stderr, "\n[block %d per warp: issued / first piece / B done / C done us]", blk);
                    for (int w = 0; w < 16; w++)
                        fprintf(stderr, " %d:%.1f/%.1f/%.1f/%.1f", w, sb[68 + w] ? (sb[68 + w] - sb[0]) * 1e-3 : -1.0,
                                sb[8 + w] ? (sb[8 + w] - sb[0]) * 1e-3 : -1.0,
                                sb[24 + w] ? (sb[24 + w] - sb[0]) * 1e-3 : -1.0,
                                sb[40 + w] ? (sb[40 + w] - sb[0]) * 1e-3 : -1.0);
                    fprintf(stderr, "\n[block %d warps 0/15: B wait/compute, C wait/compute us] %.1f/%.1f %.1f/%.1f | %.1f/%.1f %.1f/%.1f",
                            blk, sb[56] * 1e-3, sb[57] * 1e-3, sb[58] * 1e-3, sb[59] * 1e-3, sb[60] * 1e-3, sb[61] * 1e-3,
                            sb[62] * 1e-3, sb[63] * 1e-3);
                }
                fprintf(stderr, "\n");
            }
            return 0;
        }
        if (rc < 0) {
            set_err("fused decode launch failed: %s", cudaGetErrorString(cudaGetLastError()));
            return -3;
        }
        // not applicable on this device: the separate kernels below
    }
    if (a.no_routed) {
        CK(cudaMemsetAsync(rb.err, 0, sizeof(int), s));
        CK(cudaMemsetAsync(b.tc_err, 0, sizeof(int), s));
    } else {
    if (a.d_gi) {
        PhaseScope ps(kRoute, s);
        launch_router_logits(b.x, a.d_gi, T, a.E, a.n_in, rb.logits, s, rb.err);   // also zeroes err
        launch_router_select(a.rp, T, rb, s);
        g_launches += 2;
    } else {
        CK(cudaMemsetAsync(rb.err, 0, sizeof(int), s));
    }
    {
        PhaseScope ps(kDispatch, s);
        ItemLists il;
        il.zero = b.tc_err;   // status word of the expert GEMMs (both paths)
        if (b.use_tc) {
            il.gu = b.items_gu;
            il.n_gu = b.n_items;
            il.mt_gu = tc_tiles_gateup(a.inter);
            il.dn = b.items_dn;
            il.n_dn = b.n_items + 1;
            il.mt_dn = tc_tiles_down(a.n_out);
            il.tiles = b.item_tiles;
            il.nt = tc_token_tile(T * a.K, a.E);
        }
        g_launches += launch_dispatch(T, a.K, a.E, rb, s, il);
    }
    ExpertTable et{a.tab->d_w};
    const int na_max = std::min(a.E, T * a.K);
    if (b.use_tc) {
        // tensor-core path: fp16 gather, gate/up GEMM + SwiGLU, down GEMM
        static unsigned long long* stats = nullptr;   // DRACO_B200_TC_STATS=1: per-site wait cycles
        if (!stats && env_flag("DRACO_B200_TC_STATS")) {
            cudaMallocManaged(&stats, sizeof(unsigned long long) * 2 * kTcStatSites);
            cudaMemset(stats, 0, sizeof(unsigned long long) * 2 * kTcStatSites);
        }
        TcCall call;
        int rc = tc_prepare(&call, a.tab->cg, a.tab->cd, a.E, a.inter, a.n_in, a.n_out, T * a.K, b.xs_h, b.act_h);
        const TcMaps& maps = *(const TcMaps*)a.tab->tc;
        if (rc == 0) {
            PhaseScope ps(kGather, s);
            if (xh) tc_gather(call, b.x, xh, rb.ilist, rb.off + a.E, a.K, b.xs_h, s);
            else tc_gather_tokens(call, b.x, rb.order, rb.pos_of, T, a.K, a.E, b.xs_h, s);
        }
        if (rc == 0) {
            PhaseScope ps(kGateUp, s);
            rc = tc_gateup(call, maps, b.items_gu, b.n_items, b.act_h, b.tc_err, stats, s);
        }
        if (rc == 0) {
            PhaseScope ps(kDown, s);
            // expert outputs as fp16 rows: half the bytes the down GEMM writes and the combine reads
            rc = tc_down(call, maps, b.items_dn, b.n_items + 1, b.y, true, b.tc_err,
                         stats ? stats + kTcStatSites : nullptr, s);
        }
        if (stats) {
            cudaStreamSynchronize(s);
            static const char* names[kTcStatSites] = {"prod_raw_empty", "prod_b_empty", "mma_acc_empty", "mma_b_full",
                                                      "mma_a_full", "deq_raw_full", "deq_a_empty", "epi_acc_full",
                                                      "deq_total", "mma_total", "deq_decode", "deq_store", "epi_work",
                                                      "mma_test", "mma_issue"};
            for (int k = 0; k < 2; k++) {
                fprintf(stderr, "[tc stats %s]", k ? "down" : "gateup");
                for (int i = 0; i < kTcStatSites; i++) fprintf(stderr, " %s=%.3g", names[i], (double)stats[k * kTcStatSites + i]);
                fprintf(stderr, "\n");
            }
            memset(stats, 0, sizeof(unsigned long long) * 2 * kTcStatSites);
        }
        if (rc) {
            set_err("tensor-core grouped GEMM launch failed (%d): %s", rc, cudaGetErrorString(cudaGetLastError()));
            return -3;
        }
        g_launches += 3;
    } else if (g_act_mode == 0 && a.tab->aligned16 &&
               dec_supported(a.tab->cg, a.tab->cu, a.tab->cd, a.inter, a.n_in, a.n_out, a.tab->q6s)) {
        // few tokens per expert: CUDA-core GEMV over staged weight tiles
        int rc;
        {
            PhaseScope ps(kGateUp, s);
            rc = launch_dec_gateup(et, a.tab->cg, a.tab->cu, rb.active, rb.n_active, na_max, rb.off, rb.ilist, a.K,
                                   b.x, a.inter, a.n_in, b.act, a.tab->q6s, b.tc_err, s);
        }
        if (rc == 0) {
            PhaseScope ps(kDown, s);
            rc = launch_dec_down(et, a.tab->cd, rb.active, rb.n_active, na_max, rb.off, b.act, a.inter, a.n_out, b.y,
                                 a.tab->q6s, b.tc_err, s);
        }
        if (rc) {
            set_err("decode GEMV launch failed (%d): %s", rc, cudaGetErrorString(cudaGetLastError()));
            return -3;
        }
        g_launches += 2;
    } else {
    {
        PhaseScope ps(kGateUp, s);
        if (g_act_mode == 1 && a.tab->cg == a.tab->cu &&
            (a.tab->cg == DRACO_CODE_Q4_K || a.tab->cg == DRACO_CODE_Q6_K) && a.n_in % 256 == 0) {
            launch_q8k_quantize(b.x, T, a.n_in, b.xd, b.xq, b.xbs, s);
            launch_gateup_q8k(et, a.tab->cg, rb.active, rb.n_active, na_max, rb.off, rb.ilist, a.K, b.xq, b.xd,
                              b.xbs, a.inter, a.n_in, b.act, s, a.tab->q6s);
            g_launches += 2;
        } else {
            launch_gateup_codes(et, a.tab->cg, a.tab->cu, rb.active, rb.n_active, na_max, rb.off, rb.ilist, a.K,
                                b.x, a.inter, a.n_in, b.act, s, a.tab->q6s);
            g_launches += 1;
        }
    }
    {
        PhaseScope ps(kDown, s);
        launch_down_code(et, a.tab->cd, rb.active, rb.n_active, na_max, rb.off, b.act, a.inter, a.n_out, b.y, s,
                         a.tab->q6s);
        g_launches += 1;
    }
    }
    }   // routed experts
    CK(cudaGetLastError());
    if (a.sh && b.sh_tc) {
        // dense shared expert: the tensor-core GEMMs over all T token rows
        PhaseScope ps(kShared, s);
        TcCall sc;
        int rc = tc_prepare(&sc, a.sh->cg, a.sh->cd, 1, a.sh_ff, a.n_in, a.n_out, T, b.xs_h, b.act_h);
        const TcMaps& maps = *(const TcMaps*)a.sh->tc;
        if (rc == 0) {
            tc_dense_items(sc, b.items_sh_gu, b.n_items_sh, b.items_sh_dn, b.n_items_sh + 1, s);
            tc_gather(sc, b.x, xh, nullptr, nullptr, 1, b.xs_h, s);
            rc = tc_gateup(sc, maps, b.items_sh_gu, b.n_items_sh, b.act_h, b.tc_err, nullptr, s);
        }
        if (rc == 0) rc = tc_down(sc, maps, b.items_sh_dn, b.n_items_sh + 1, b.y_sh, false, b.tc_err, nullptr, s);
        if (rc) {
            set_err("shared-expert tensor-core GEMM launch failed (%d)", rc);
            return -3;
        }
        g_launches += 4;
    } else if (a.sh) {
        if (int rc = dense_ffn(c, a.sh, T, b.x, a.sh_ff, a.n_in, a.n_out, b.act_sh, b.y_sh, b.tc_err, s)) return rc;
    }
    {
        PhaseScope ps(kCombine, s);
        if (b.use_tc && !a.no_routed)
            launch_combine_half(reinterpret_cast<const __half*>(b.y), rb.order, rb.wtop, rb.pos_of, T, a.K, a.E,
                                a.n_out, a.sh ? b.y_sh : nullptr, b.out, s, a.out_blk, a.out_block);
        else
            launch_combine(b.y, rb.order, rb.wtop, rb.pos_of, T, a.no_routed ? 0 : a.K, a.E, a.n_out,
                           a.sh ? b.y_sh : nullptr, b.out, s, a.out_blk, a.out_block);
        g_launches += 1;
    }
    CK(cudaGetLastError());
    return 0;
}

int check_route_err(Ctx* c, LayerBufs& b, cudaStream_t s) {
    int h_err = 0, h_tc = 0;
    CK(cudaMemcpyAsync(&h_err, b.rb.err, sizeof(int), cudaMemcpyDeviceToHost, s));
    CK(cudaMemcpyAsync(&h_tc, b.tc_err, sizeof(int), cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    if (h_tc) {
        set_err("expert GEMM stopped after a bounded wait ran out (code 0x%x)", h_tc);
        return -5;
    }
    if (h_err) {
        set_err("routing found fewer eligible experts than n_used (group limit or non-finite scores), code %d",
                h_err);
        return -2;
    }
    return 0;
}

int validate_shape(int n_exp, int n_used, int inter, int n_in, int n_out, int n_group, int n_group_used) {
    if (n_exp <= 0 || n_exp > 512 || n_used <= 0 || n_used > 64 || n_used > n_exp || inter <= 0 || n_in <= 0 ||
        n_out <= 0) {
        set_err("unsupported shape n_exp=%d n_used=%d inter=%d n_in=%d n_out=%d (need 1<=n_used<=64, "
                "n_used<=n_exp<=512)", n_exp, n_used, inter, n_in, n_out);
        return -1;
    }
    if (n_group > 1 && (n_group > 64 || n_exp % n_group || n_group_used < 1 || n_group_used > n_group ||
                        n_group_used * (n_exp / n_group) < n_used)) {
        set_err("unsupported grouping n_group=%d n_group_used=%d for n_exp=%d n_used=%d", n_group, n_group_used,
                n_exp, n_used);
        return -1;
    }
    return 0;
}

uint32_t __float_as_uint_host(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}

// Run `body` (launches on stream s) through a cached CUDA graph keyed by `key`: capture it on
// the first call, replay it afterwards.  Falls back to direct launches while profiling, when
// the caller is itself capturing the stream, or when capture fails.
template <class F>
int graph_call(Ctx* c, const std::vector<uint64_t>& key, cudaStream_t s, F&& body) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (g_prof || env_flag("DRACO_B200_TC_STATS") || env_flag("DRACO_B200_NO_GRAPH") ||
        cudaStreamIsCapturing(s, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
        cudaGetLastError();
        return body();
    }
    for (auto& g : c->graphs)
        if (g.key == key) {
            g.last_use = ++c->graph_clock;
            CK(cudaGraphLaunch(g.exec, s));
            g_launches += g.launches;
            return 0;
        }
    if (cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        cudaGetLastError();
        return body();
    }
    const long l0 = g_launches;
    const int rc = body();
    cudaGraph_t graph = nullptr;
    const cudaError_t ec = cudaStreamEndCapture(s, &graph);
    cudaGraphExec_t exec = nullptr;
    if (rc == 0 && ec == cudaSuccess && graph && cudaGraphInstantiate(&exec, graph, 0) == cudaSuccess) {
        cudaGraphDestroy(graph);
        Ctx::Graph g;
        g.key = key;
        g.exec = exec;
        g.launches = g_launches - l0;
        g.last_use = ++c->graph_clock;
        if (c->graphs.size() >= 16) {   // evict the least recently used
            auto lru = std::min_element(c->graphs.begin(), c->graphs.end(),
                                        [](const Ctx::Graph& x, const Ctx::Graph& y) { return x.last_use < y.last_use; });
            cudaGraphExecDestroy(lru->exec);
            c->graphs.erase(lru);
        }
        c->graphs.push_back(std::move(g));
        g_launches = l0;
        CK(cudaGraphLaunch(exec, s));
        g_launches += c->graphs.back().launches;
        return 0;
    }
    if (graph) cudaGraphDestroy(graph);
    cudaGetLastError();
    g_launches = l0;
    if (rc) return rc;
    return body();   // capture failed: launch directly
}

// Synchronous single-call layer on host or device x/out (the reference entry points).
int layer_call(const float* x, int T, const uint64_t* ptrs, const int* codes, const float* gate_inp,
               const float* probs_b, int scoring, int n_exp, int n_used, int n_group, int n_group_used, int norm_w,
               float w_scale, int inter, int n_in, int n_out, const uint64_t* sh3, const int* shc3, int sh_ff,
               float* out, int* order_out, float* wtop_out, cudaStream_t user_stream,
               const GivenRoute* gr = nullptr) {
    // gr given: the routing is the caller's and gate_inp is not used
    if (int rc = validate_shape(n_exp, n_used, inter, n_in, n_out, scoring ? n_group : 1, n_group_used)) return rc;
    if (T <= 0) return 0;
    Ctx* c = get_ctx();
    if (!c) return -3;
    const double t0 = now_s();
    LayerArgs a;
    a.E = n_exp;
    a.K = n_used;
    a.inter = inter;
    a.n_in = n_in;
    a.n_out = n_out;
    // resolve every weight range; an upload that replaced a changed range drops cached
    // tables, so repeat until one pass completes without that
    unsigned long gen0 = 0;
    for (int attempt = 0; attempt < 3; attempt++) {
        gen0 = c->gen;
        a.d_gi = nullptr;
        if (!gr) {
            a.d_gi = (const float*)dev_range(c, gate_inp, sizeof(float) * (size_t)n_exp * n_in);
            if (!a.d_gi) return -1;
        }
        a.rp.probs_b = nullptr;
        if (!gr && scoring && probs_b) {
            a.rp.probs_b = (const float*)dev_range(c, probs_b, sizeof(float) * n_exp);
            if (!a.rp.probs_b) return -1;
        }
        a.tab = get_table(c, ptrs, codes, n_exp, inter, n_in, n_out);
        if (!a.tab) return -1;
        a.sh = nullptr;
        if (sh3 && sh_ff > 0) {
            a.sh = get_table(c, sh3, shc3, 1, sh_ff, n_in, n_out, (uintptr_t)sh3[0]);
            if (!a.sh) return -1;
            a.sh_ff = sh_ff;
        }
        if (c->gen == gen0) break;
    }
    if (c->gen != gen0) {
        set_err("weight ranges keep changing under the call");
        return -1;
    }
    a.rp.scoring = scoring;
    a.rp.n_exp = n_exp;
    a.rp.n_used = n_used;
    a.rp.n_in = n_in;
    a.rp.n_group = scoring ? n_group : 1;
    a.rp.n_group_used = n_group_used;
    a.rp.norm_w = norm_w;
    a.rp.w_scale = w_scale;
    a.no_routed = gr && !gr->order;
    a.x_half = gr && gr->x_half;
    if (gr && gr->out_blk) {
        a.out_blk = gr->out_blk;
        a.out_block = gr->out_block;
    }
    if (a.no_routed && !a.sh) {
        set_err("no routed experts and no shared expert: nothing to compute");
        return -1;
    }
    LayerBufs b;
    if (int rc = carve_layer(c, a, T, b)) return rc;
    const bool dev_io = dev_kind(x);
    if (dev_io && ((uintptr_t)x & 15 || (uintptr_t)out & 15)) {
        set_err("device activations and outputs must be 16-byte aligned");
        return -1;
    }
    if (a.x_half && !dev_io) {
        set_err("fp16 activation rows must be device memory");
        return -1;
    }
    if (gr && gr->order && (dev_kind(gr->order) != dev_io || dev_kind(gr->wtop) != dev_io)) {
        set_err("order and wtop must live where the activations live (all host or all device)");
        return -1;
    }
    cudaStream_t s = (dev_io && user_stream) ? user_stream : c->stream;
    if (dev_io && !user_stream)
        if (int rc = after_legacy_stream(c)) return rc;
    // a stream being captured by the caller: no ordering against work outside the capture
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &cap) != cudaSuccess) cudaGetLastError();
    const bool captured = cap != cudaStreamCaptureStatusNone;
    if (captured) c->ws_captured = true;
    else ws_acquire(c, s);
    float* d_out = b.out;
    if (dev_io) {
        b.x = const_cast<float*>(x);
        d_out = out;
        b.out = out;
    }
    auto body = [&]() -> int {
        if (gr && gr->order) {
            if (dev_io) {
                launch_route_in(gr->order, gr->wtop, gr->ld, gr->e_base, T, n_used, b.rb.order, b.rb.wtop, s);
                g_launches += 1;
            } else {
                const size_t w = sizeof(int) * n_used, ld = sizeof(int) * gr->ld;
                CK(cudaMemcpy2DAsync(b.rb.order, w, gr->order, ld, w, T, cudaMemcpyHostToDevice, s));
                CK(cudaMemcpy2DAsync(b.rb.wtop, w, gr->wtop, ld, w, T, cudaMemcpyHostToDevice, s));
                if (gr->e_base) {
                    launch_route_in(b.rb.order, b.rb.wtop, n_used, gr->e_base, T, n_used, b.rb.order, b.rb.wtop, s);
                    g_launches += 1;
                }
            }
        }
        if (int rc = run_layer(c, a, T, b, s)) return rc;
        if (dev_io) {
            if (order_out)
                CK(cudaMemcpyAsync(order_out, b.rb.order, sizeof(int) * T * n_used, cudaMemcpyDeviceToDevice, s));
            if (wtop_out)
                CK(cudaMemcpyAsync(wtop_out, b.rb.wtop, sizeof(float) * T * n_used, cudaMemcpyDeviceToDevice, s));
        }
        return 0;
    };
    if (dev_io && user_stream) {
        // asynchronous call: replay the captured launch sequence of an identical earlier call
        const std::vector<uint64_t> key = {
            (uintptr_t)a.tab, (uintptr_t)a.sh, c->gen, (uintptr_t)c->ws, c->ws_cap, (uintptr_t)a.d_gi,
            (uintptr_t)a.rp.probs_b, (uintptr_t)x, (uintptr_t)out, (uintptr_t)order_out, (uintptr_t)wtop_out,
            (uint64_t)T, (uintptr_t)s, (uint64_t)n_exp, (uint64_t)n_used, (uint64_t)inter, (uint64_t)n_in,
            (uint64_t)n_out, (uint64_t)a.sh_ff, (uint64_t)a.rp.scoring, (uint64_t)a.rp.n_group,
            (uint64_t)a.rp.n_group_used, (uint64_t)a.rp.norm_w, (uint64_t)__float_as_uint_host(a.rp.w_scale),
            (uint64_t)gemm_path(), (uint64_t)g_act_mode, (uint64_t)b.use_tc, (uint64_t)(gr != nullptr),
            (uintptr_t)(gr ? gr->order : nullptr), (uintptr_t)(gr ? gr->wtop : nullptr), (uint64_t)(gr ? gr->ld : 0),
            (uint64_t)(gr ? gr->e_base : 0), (uint64_t)a.x_half, (uintptr_t)a.out_blk, (uint64_t)a.out_block};
        const int rc = captured ? body() : graph_call(c, key, s, body);
        if (!captured) ws_release(c, s);
        return rc;
    }
    // synchronous call on page-locked host buffers: the copies and the launches replay as one
    // captured graph; the status words come back through the context's page-locked buffer
    const bool host_graph = !dev_io && !captured && !gr && host_graph_enabled() && is_pinned_host(x) &&
                            is_pinned_host(out) && (!order_out || is_pinned_host(order_out)) &&
                            (!wtop_out || is_pinned_host(wtop_out));
    if (host_graph) {
        auto body_h = [&]() -> int {
            if (int rc = h2d(c, b.x, x, sizeof(float) * (size_t)T * n_in, s)) return rc;
            if (int rc = body()) return rc;
            CK(cudaMemcpyAsync(out, d_out, sizeof(float) * (size_t)T * n_out, cudaMemcpyDeviceToHost, s));
            if (order_out) CK(cudaMemcpyAsync(order_out, b.rb.order, sizeof(int) * T * n_used, cudaMemcpyDeviceToHost, s));
            if (wtop_out) CK(cudaMemcpyAsync(wtop_out, b.rb.wtop, sizeof(float) * T * n_used, cudaMemcpyDeviceToHost, s));
            CK(cudaMemcpyAsync(c->h_status, b.rb.err, sizeof(int), cudaMemcpyDeviceToHost, s));
            CK(cudaMemcpyAsync(c->h_status + 1, b.tc_err, sizeof(int), cudaMemcpyDeviceToHost, s));
            return 0;
        };
        const std::vector<uint64_t> key = {
            2, (uintptr_t)a.tab, (uintptr_t)a.sh, c->gen, (uintptr_t)c->ws, c->ws_cap, (uintptr_t)a.d_gi,
            (uintptr_t)a.rp.probs_b, (uintptr_t)x, (uintptr_t)out, (uintptr_t)order_out, (uintptr_t)wtop_out,
            (uint64_t)T, (uintptr_t)s, (uint64_t)n_exp, (uint64_t)n_used, (uint64_t)inter, (uint64_t)n_in,
            (uint64_t)n_out, (uint64_t)a.sh_ff, (uint64_t)a.rp.scoring, (uint64_t)a.rp.n_group,
            (uint64_t)a.rp.n_group_used, (uint64_t)a.rp.norm_w, (uint64_t)__float_as_uint_host(a.rp.w_scale),
            (uint64_t)gemm_path(), (uint64_t)g_act_mode, (uint64_t)b.use_tc, (uint64_t)fused_decode_enabled()};
        if (int rc = graph_call(c, key, s, body_h)) return rc;
        ws_release(c, s);
        CK(cudaStreamSynchronize(s));
        const int h_err = c->h_status[0], h_tc = c->h_status[1];
        if (h_tc) {
            set_err("expert GEMM stopped after a bounded wait ran out (code 0x%x)", h_tc);
            return -5;
        }
        if (h_err) {
            set_err("routing found fewer eligible experts than n_used (group limit or non-finite scores), code %d",
                    h_err);
            return -2;
        }
        m6_prof_t[23] += now_s() - t0;
        m6_prof_n[23]++;
        return 0;
    }
    if (!dev_io) {
        if (int rc = h2d(c, b.x, x, sizeof(float) * (size_t)T * n_in, s)) return rc;
    }
    if (int rc = body()) return rc;
    if (dev_io) {
        if (!captured) ws_release(c, s);
        if (user_stream) return 0;
    } else {
        CK(cudaMemcpyAsync(out, d_out, sizeof(float) * (size_t)T * n_out, cudaMemcpyDeviceToHost, s));
        if (order_out) CK(cudaMemcpyAsync(order_out, b.rb.order, sizeof(int) * T * n_used, cudaMemcpyDeviceToHost, s));
        if (wtop_out) CK(cudaMemcpyAsync(wtop_out, b.rb.wtop, sizeof(float) * T * n_used, cudaMemcpyDeviceToHost, s));
    }
    if (int rc = check_route_err(c, b, s)) return rc;
    m6_prof_t[23] += now_s() - t0;
    m6_prof_n[23]++;
    return 0;
}

template <typename T>
int stage_in(Ctx* c, cudaStream_t s, size_t off, const T* h, size_t n) {
    CK(cudaMemcpyAsync(c->ws + off, h, sizeof(T) * n, cudaMemcpyHostToDevice, s));
    return 0;
}

}  // namespace

// ===================================== Part 1 ==========================================
extern "C" {

void m6_granite_moe(const float* x0, const uint64_t* ptrs, const int* codes, const float* gate_inp, int n_exp,
                    int n_used, int inter, int n_in, int n_out, float* scratch, float* out) {
    (void)scratch;
    std::lock_guard<std::mutex> lk(g_mu);
    if (layer_call(x0, 1, ptrs, codes, gate_inp, nullptr, 0, n_exp, n_used, 1, 1, 1, 0.f, inter, n_in, n_out,
                   nullptr, nullptr, 0, out, nullptr, nullptr, nullptr))
        fail_void("m6_granite_moe", out, (size_t)(n_out > 0 ? n_out : 0));
}

void m6_bailing_moe(const float* x0, const uint64_t* ptrs, const int* codes, const float* gate_inp,
                    const float* probs_b, int n_exp, int n_used, int n_group, int n_group_used, int norm_w,
                    float w_scale, int inter, int n_in, int n_out, float* scratch, float* out) {
    (void)scratch;
    std::lock_guard<std::mutex> lk(g_mu);
    if (layer_call(x0, 1, ptrs, codes, gate_inp, probs_b, 1, n_exp, n_used, n_group, n_group_used, norm_w, w_scale,
                   inter, n_in, n_out, nullptr, nullptr, 0, out, nullptr, nullptr, nullptr))
        fail_void("m6_bailing_moe", out, (size_t)(n_out > 0 ? n_out : 0));
}

void m6_moe_op(const float* xn, void* pv, float* out) {
    std::lock_guard<std::mutex> lk(g_mu);
    const M6MoeP* p = (const M6MoeP*)pv;
    const uint64_t sh3[3] = {(uint64_t)(uintptr_t)p->sh_g, (uint64_t)(uintptr_t)p->sh_u,
                             (uint64_t)(uintptr_t)p->sh_d};
    const int shc3[3] = {p->csg, p->csu, p->csd};
    const bool has_sh = p->sh_g && p->sh_u && p->sh_d && p->sh_ff > 0;
    if (layer_call(xn, 1, p->exp_ptrs, p->exp_codes, p->gate_inp, p->probs_b, 1, p->n_exp, p->n_used, p->n_group,
                   p->n_group_used, p->norm_w, p->w_scale, p->inter, p->n_in, p->n_out, has_sh ? sh3 : nullptr,
                   shc3, has_sh ? p->sh_ff : 0, out, nullptr, nullptr, nullptr))
        fail_void("m6_moe_op", out, (size_t)(p->n_out > 0 ? p->n_out : 0));
}

static int shexp_impl(const float* x, const uint64_t* shp, const int* shc, float* sg, float* shg, float* out, int shi,
                      int h) {
    if (shc[3] != DRACO_CODE_F32) {
        set_err("shared-expert gate row format %d unsupported (F32 = 9 expected)", shc[3]);
        return -1;
    }
    Ctx* c = get_ctx();
    if (!c) return -3;
    const float* gw = (const float*)dev_range(c, (const void*)(uintptr_t)shp[3], sizeof(float) * h);
    if (!gw) return -1;
    const unsigned long gen0 = c->gen;
    Table* t = get_table(c, shp, shc, 1, shi, h, h, (uintptr_t)shp[0]);
    if (!t) return -1;
    if (c->gen != gen0) {   // the table upload replaced a range: resolve the gate row again
        gw = (const float*)dev_range(c, (const void*)(uintptr_t)shp[3], sizeof(float) * h);
        t = get_table(c, shp, shc, 1, shi, h, h, (uintptr_t)shp[0]);
        if (!gw || !t) return -1;
    }
    Carver cv;
    const size_t o_x = cv.take<float>(h), o_a = cv.take<float>(shi), o_y = cv.take<float>(h);
    const size_t o_o = cv.take<float>(h), o_sg = cv.take<float>(1);
    if (int rc = ensure_ws(c, cv.off)) return rc;
    float* dx = (float*)(c->ws + o_x);
    float* da = (float*)(c->ws + o_a);
    float* dy = (float*)(c->ws + o_y);
    float* dout = (float*)(c->ws + o_o);
    float* dsg = (float*)(c->ws + o_sg);
    cudaStream_t s = c->stream;
    CK(cudaMemcpyAsync(dx, x, sizeof(float) * h, cudaMemcpyHostToDevice, s));
    if (int rc = dense_ffn(c, t, 1, dx, shi, h, h, da, dy, nullptr, s)) return rc;
    launch_shexp_gate(dx, gw, h, dy, dsg, dout, 1, s);
    CK(cudaGetLastError());
    CK(cudaMemcpyAsync(out, dout, sizeof(float) * h, cudaMemcpyDeviceToHost, s));
    if (sg) CK(cudaMemcpyAsync(sg, dsg, sizeof(float), cudaMemcpyDeviceToHost, s));
    if (shg) CK(cudaMemcpyAsync(shg, dy, sizeof(float) * h, cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    return 0;
}

void m6_granite_shexp(const float* x, const uint64_t* shp, const int* shc, float* sg, float* sh, float* shg,
                      float* out, int shi, int h) {
    (void)sh;
    std::lock_guard<std::mutex> lk(g_mu);
    if (shexp_impl(x, shp, shc, sg, shg, out, shi, h)) fail_void("m6_granite_shexp", out, (size_t)(h > 0 ? h : 0));
}

static int moe_tok_impl(const float* X, const int* order, const float* wtop, const uint64_t* ep, const int* ec, int T,
                        int n_used, int inter, int n_in, int n_out, int n_exp, float* out) {
    if (int rc = validate_shape(n_exp, n_used, inter, n_in, n_out, 1, 1)) return rc;
    if (T <= 0) return 0;
    Ctx* c = get_ctx();
    if (!c) return -3;
    const double t0 = now_s();
    LayerArgs a;
    a.E = n_exp;
    a.K = n_used;
    a.inter = inter;
    a.n_in = n_in;
    a.n_out = n_out;
    a.tab = get_table(c, ep, ec, n_exp, inter, n_in, n_out);
    if (!a.tab) return -1;
    LayerBufs b;
    if (int rc = carve_layer(c, a, T, b)) return rc;
    cudaStream_t s = c->stream;
    const size_t n = (size_t)T * n_used;
    const bool dev_io = dev_kind(X);
    if (dev_io && ((uintptr_t)X & 15 || (uintptr_t)out & 15)) {
        set_err("device activations and outputs must be 16-byte aligned");
        return -1;
    }
    if (dev_io) {
        if (int rc = after_legacy_stream(c)) return rc;
        b.x = const_cast<float*>(X);
        b.out = out;
        CK(cudaMemcpyAsync(b.rb.order, order, sizeof(int) * n, cudaMemcpyDeviceToDevice, s));
        CK(cudaMemcpyAsync(b.rb.wtop, wtop, sizeof(float) * n, cudaMemcpyDeviceToDevice, s));
    } else {
        if (int rc = h2d(c, b.x, X, sizeof(float) * (size_t)T * n_in, s)) return rc;
        CK(cudaMemcpyAsync(b.rb.order, order, sizeof(int) * n, cudaMemcpyHostToDevice, s));
        CK(cudaMemcpyAsync(b.rb.wtop, wtop, sizeof(float) * n, cudaMemcpyHostToDevice, s));
    }
    if (int rc = run_layer(c, a, T, b, s)) return rc;
    if (!dev_io) CK(cudaMemcpyAsync(out, b.out, sizeof(float) * (size_t)T * n_out, cudaMemcpyDeviceToHost, s));
    CK(cudaMemsetAsync(b.rb.err, 0, sizeof(int), s));   // routing was given: only the GEMM status counts
    if (int rc = check_route_err(c, b, s)) return rc;
    m6_prof_t[23] += now_s() - t0;
    m6_prof_n[23]++;
    return 0;
}

void m6_moe_tok(m6_dequant_fn DQ, m6_gemm_auto_fn GA, float* gwbuf, const float* X, const int* order,
                const float* wtop, const uint64_t* ep, const int* ec, int T, int n_used, int inter, int n_in,
                int n_out, int n_exp, float* out, float* work, int* iwork) {
    (void)DQ;
    (void)GA;
    (void)gwbuf;
    (void)work;
    (void)iwork;
    std::lock_guard<std::mutex> lk(g_mu);
    if (moe_tok_impl(X, order, wtop, ep, ec, T, n_used, inter, n_in, n_out, n_exp, out))
        fail_void("m6_moe_tok", dev_kind(out) ? nullptr : out, (size_t)(T > 0 && n_out > 0 ? (size_t)T * n_out : 0));
}

// ---- caller-routed single-token variants (src/m6_layer.c:520-690): the table holds exactly the
// n_exp selected experts, wtop their weights; out = sum_j wtop[j] * expert_j(x0), j ascending
static int moe_batch_impl(const float* x0, const uint64_t* ptrs, const int* codes, const float* wtop, int n_exp,
                          int inter, int n_in, int n_out, float* out) {
    if (n_exp <= 0 || n_exp > 64) {
        set_err("m6_moe_batch: 1 <= n_exp <= 64 selected experts expected, got %d", n_exp);
        return -1;
    }
    int order[64];
    for (int j = 0; j < n_exp; j++) order[j] = j;
    return moe_tok_impl(x0, order, wtop, ptrs, codes, 1, n_exp, inter, n_in, n_out, n_exp, out);
}

void m6_moe_batch(const float* x0, const uint64_t* ptrs, const int* codes, const float* wtop, int n_exp, float* out) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (moe_batch_impl(x0, ptrs, codes, wtop, n_exp, 512, 2048, 2048, out)) fail_void("m6_moe_batch", out, 2048);
}

void m6_moe_batch2(const float* x0, const uint64_t* ptrs, const int* codes, const float* wtop, int n_exp,
                   const uint64_t* sh_ptrs, const int* sh_codes, const float* sh_gate_inp, float* scratch,
                   float* out) {
    (void)scratch;
    std::lock_guard<std::mutex> lk(g_mu);
    int rc = moe_batch_impl(x0, ptrs, codes, wtop, n_exp, 512, 2048, 2048, out);
    // + sigmoid(x0 . sh_gate_inp) * shared expert; without a gate row the reference's gate is 0
    if (rc == 0 && sh_gate_inp && sh_ptrs && sh_codes) {
        const uint64_t shp[4] = {sh_ptrs[0], sh_ptrs[1], sh_ptrs[2], (uint64_t)(uintptr_t)sh_gate_inp};
        const int shc[4] = {sh_codes[0], sh_codes[1], sh_codes[2], DRACO_CODE_F32};
        std::vector<float> g(2048);
        rc = shexp_impl(x0, shp, shc, nullptr, nullptr, g.data(), 512, 2048);
        if (rc == 0)
            for (int i = 0; i < 2048; i++) out[i] += g[i];
    }
    if (rc) fail_void("m6_moe_batch2", out, 2048);
}

void m6_moe_batch3(const float* x0, const uint64_t* ptrs, const int* codes, const float* wtop, int n_exp, int inter,
                   int n_in, int n_out, float* out) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (moe_batch_impl(x0, ptrs, codes, wtop, n_exp, inter, n_in, n_out, out))
        fail_void("m6_moe_batch3", out, (size_t)(n_out > 0 ? n_out : 0));
}

void m6_moe_batch4(const float* x0, const uint64_t* ptrs, const int* codes, const float* wtop, int n_exp, int inter,
                   int n_in, int n_out, float* scratch, float* out) {
    (void)scratch;
    std::lock_guard<std::mutex> lk(g_mu);
    if (moe_batch_impl(x0, ptrs, codes, wtop, n_exp, inter, n_in, n_out, out))
        fail_void("m6_moe_batch4", out, (size_t)(n_out > 0 ? n_out : 0));
}

// ---- top-1 MoE with a learned router MLP (src/m6_engine.c:795-835) ----
static int zaya_impl(const float* xn, const M6ZayaMoeP* p, float* out) {
    const int H = p->hidden, RH = p->hidden2, F = p->inter, NE = p->nexp;
    if (H <= 0 || RH <= 0 || F <= 0 || NE <= 0 || NE > 512 || p->nclass <= 0 || p->nclass > 1024) {
        set_err("m6_zaya_moe_op: unsupported shape hidden=%d hidden2=%d inter=%d nexp=%d nclass=%d", H, RH, F, NE,
                p->nclass);
        return -1;
    }
    auto f16or32 = [](int c) { return c == 9 || c == 7; };
    if (!f16or32(p->cdown) || !f16or32(p->cfc1) || !f16or32(p->cfc2) || !f16or32(p->cout)) {
        set_err("m6_zaya_moe_op: router matrices must be F32 (9) or F16 (7)");
        return -1;
    }
    Ctx* c = get_ctx();
    if (!c) return -3;
    const double t0 = now_s();
    const int cg = p->exp_cg[0], cd = p->exp_cd[0];
    const size_t rbg = row_bytes(cg, H);
    std::vector<uint64_t> ep(3 * (size_t)NE);
    std::vector<int> ec(3 * (size_t)NE);
    for (int e = 0; e < NE; e++) {
        if (p->exp_cg[e] != cg || p->exp_cd[e] != cd) {
            set_err("m6_zaya_moe_op: experts with different formats are unsupported");
            return -1;
        }
        // the fused gate|up matrix of 2*inter rows: gate rows first, then up
        ep[3 * e] = p->exp_gp[e];
        ep[3 * e + 1] = p->exp_gp[e] + (uint64_t)F * rbg;
        ep[3 * e + 2] = p->exp_dp[e];
        ec[3 * e] = ec[3 * e + 1] = cg;
        ec[3 * e + 2] = cd;
    }
    auto esz = [](int code) { return code == 9 ? 4 : 2; };
    ZayaRouterArgs z{};
    LayerArgs a;
    a.E = NE;
    a.K = 1;
    a.inter = F;
    a.n_in = H;
    a.n_out = H;
    unsigned long gen0 = 0;
    for (int attempt = 0; attempt < 3; attempt++) {
        gen0 = c->gen;
        // the whole fused gate|up tensors first (gate and up halves then resolve inside them):
        // one range when the experts are stacked (base + e * per), else one per expert
        if (cg != DRACO_CODE_Q6_K) {
            const uint64_t base = p->exp_gp[0], per = NE > 1 ? p->exp_gp[1] - base : 0;
            bool stacked = NE > 1 && p->exp_gp[1] > base && per >= 2 * (uint64_t)F * rbg;
            for (int e = 2; stacked && e < NE; e++) stacked = p->exp_gp[e] == base + per * (uint64_t)e;
            if (stacked) {
                if (!dev_range(c, (const void*)(uintptr_t)base, per * (NE - 1) + 2 * (size_t)F * rbg)) return -1;
            } else {
                for (int e = 0; e < NE; e++)
                    if (!dev_range(c, (const void*)(uintptr_t)p->exp_gp[e], 2 * (size_t)F * rbg)) return -1;
            }
        }
        z.wdown = dev_range(c, p->wdown, (size_t)RH * H * esz(p->cdown));
        z.wfc1 = dev_range(c, p->wfc1, (size_t)RH * RH * esz(p->cfc1));
        z.wfc2 = dev_range(c, p->wfc2, (size_t)RH * RH * esz(p->cfc2));
        z.wout = dev_range(c, p->wout, (size_t)p->nclass * RH * esz(p->cout));
        z.bdown = (const float*)dev_range(c, p->bdown, sizeof(float) * RH);
        z.bfc1 = (const float*)dev_range(c, p->bfc1, sizeof(float) * RH);
        z.bfc2 = (const float*)dev_range(c, p->bfc2, sizeof(float) * RH);
        z.rnorm = (const float*)dev_range(c, p->rnorm, sizeof(float) * RH);
        z.bal = (const float*)dev_range(c, p->bal, sizeof(float) * p->nclass);
        z.eda_scale = p->eda_scale ? (const float*)dev_range(c, p->eda_scale, sizeof(float) * RH) : nullptr;
        if (!z.wdown || !z.wfc1 || !z.wfc2 || !z.wout || !z.bdown || !z.bfc1 || !z.bfc2 || !z.rnorm || !z.bal ||
            (p->eda_scale && !z.eda_scale))
            return -1;
        a.tab = get_table(c, ep.data(), ec.data(), NE, F, H, H, (uintptr_t)p->exp_gp);
        if (!a.tab) return -1;
        if (c->gen == gen0) break;
    }
    if (c->gen != gen0) {
        set_err("weight ranges keep changing under the call");
        return -1;
    }
    LayerBufs b;
    size_t o_z = 0;   // router scratch: state in, state out, rh
    if (int rc = carve_layer(c, a, 1, b, 3 * align_up(sizeof(float) * RH, 256), &o_z)) return rc;
    float* d_si = (float*)(c->ws + o_z);
    float* d_so = (float*)(c->ws + o_z + align_up(sizeof(float) * RH, 256));
    cudaStream_t s = c->stream;
    CK(cudaMemcpyAsync(b.x, xn, sizeof(float) * H, cudaMemcpyHostToDevice, s));
    if (p->eda_scale) CK(cudaMemcpyAsync(d_si, p->rh_state, sizeof(float) * RH, cudaMemcpyHostToDevice, s));
    z.cdown = p->cdown;
    z.cfc1 = p->cfc1;
    z.cfc2 = p->cfc2;
    z.cout = p->cout;
    z.x = b.x;
    z.state_in = d_si;
    z.state_out = d_so;
    z.rh = (float*)(c->ws + o_z + 2 * align_up(sizeof(float) * RH, 256));
    z.H = H;
    z.RH = RH;
    z.nclass = p->nclass;
    z.nexp = NE;
    z.iskip = p->iskip;
    z.order = b.rb.order;
    z.wtop = b.rb.wtop;
    if (launch_zaya_router(z, s)) {
        set_err("m6_zaya_moe_op: router launch failed: %s", cudaGetErrorString(cudaGetLastError()));
        return -3;
    }
    g_launches += 2;
    if (int rc = run_layer(c, a, 1, b, s)) return rc;
    CK(cudaMemcpyAsync(out, b.out, sizeof(float) * H, cudaMemcpyDeviceToHost, s));
    CK(cudaMemcpyAsync(p->rh_state, d_so, sizeof(float) * RH, cudaMemcpyDeviceToHost, s));
    CK(cudaMemsetAsync(b.rb.err, 0, sizeof(int), s));   // routing came from the router MLP
    if (int rc = check_route_err(c, b, s)) return rc;
    m6_prof_t[23] += now_s() - t0;
    m6_prof_n[23]++;
    return 0;
}

void m6_zaya_moe_op(const float* xn, void* pv, float* out) {
    std::lock_guard<std::mutex> lk(g_mu);
    const M6ZayaMoeP* p = (const M6ZayaMoeP*)pv;
    if (!p || zaya_impl(xn, p, out)) fail_void("m6_zaya_moe_op", out, p && p->hidden > 0 ? (size_t)p->hidden : 0);
}

static int gemvn_impl(int code, const float* x, long x_stride, const uint8_t* W, const int* idx, long per,
                      int n_out_e, int n_in, int n_exp, float* y) {
    const int nb = n_in / 256;
    if (nb <= 0 || n_in % 256 != 0 || (code == DRACO_CODE_Q4_K && nb > 256)) {
        set_err("m5_gemvn: n_in %d must be a positive multiple of 256", n_in);
        return -1;
    }
    if (n_exp <= 0 || n_out_e <= 0) return 0;
    Ctx* c = get_ctx();
    if (!c) return -3;
    const size_t xn = x_stride ? (size_t)x_stride * (n_exp - 1) + n_in : (size_t)n_in;
    Carver cv;
    const size_t o_x = cv.take<float>(xn), o_y = cv.take<float>((size_t)n_exp * n_out_e);
    if (int rc = ensure_ws(c, cv.off)) return rc;
    float* dx = (float*)(c->ws + o_x);
    float* dy = (float*)(c->ws + o_y);
    cudaStream_t s = c->stream;
    CK(cudaMemcpyAsync(dx, x, sizeof(float) * xn, cudaMemcpyHostToDevice, s));
    for (int e = 0; e < n_exp; e++) {
        size_t dp = 0;
        const uint8_t* dw = dev_matrix(c, W + (size_t)idx[e] * per, code, n_out_e, n_in, 1, 0, &dp);
        if (!dw) return -3;
        launch_gemv_rows(code, dw, dx + (size_t)e * x_stride, n_in, 0, n_out_e, dy + (size_t)e * n_out_e, s,
                         kQ6Padded);
    }
    CK(cudaGetLastError());
    CK(cudaMemcpyAsync(y, dy, sizeof(float) * (size_t)n_exp * n_out_e, cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    return 0;
}

int m5_gemvn_q4k(const float* x, long x_stride, const uint8_t* W, const int* idx, long per, int n_out_e, int n_in,
                 int n_exp, float* y) {
    std::lock_guard<std::mutex> lk(g_mu);
    return gemvn_impl(DRACO_CODE_Q4_K, x, x_stride, W, idx, per, n_out_e, n_in, n_exp, y);
}

int m5_gemvn_q6k(const float* x, long x_stride, const uint8_t* W, const int* idx, long per, int n_out_e, int n_in,
                 int n_exp, float* y) {
    std::lock_guard<std::mutex> lk(g_mu);
    return gemvn_impl(DRACO_CODE_Q6_K, x, x_stride, W, idx, per, n_out_e, n_in, n_exp, y);
}

int m5_scalar_supported(int code) { return code_supported(code) ? 1 : 0; }

static int gemm_impl(int code, const float* X, const uint8_t* W, int T, int n_out, int n_in, float* Y, int o0,
                     int o1) {
    if (!code_supported(code)) {
        set_err("unsupported format code %d", code);
        return -1;
    }
    if (n_in % block_values(code) || (code != DRACO_CODE_Q8_0 && n_in % 256)) {
        set_err("n_in %d not a multiple of the block size", n_in);
        return -1;
    }
    if (T <= 0 || o1 <= o0) return 0;
    Ctx* c = get_ctx();
    if (!c) return -3;
    size_t dp = 0;
    const uint8_t* dw = dev_matrix(c, W, code, n_out, n_in, 1, 0, &dp);
    if (!dw) return -3;
    Carver cv;
    const size_t o_x = cv.take<float>((size_t)T * n_in), o_y = cv.take<float>((size_t)T * n_out);
    if (int rc = ensure_ws(c, cv.off)) return rc;
    float* dx = (float*)(c->ws + o_x);
    float* dy = (float*)(c->ws + o_y);
    cudaStream_t s = c->stream;
    CK(cudaMemcpyAsync(dx, X, sizeof(float) * (size_t)T * n_in, cudaMemcpyHostToDevice, s));
    if (T == 1) {
        launch_gemv_rows(code, dw, dx, n_in, o0, o1, dy, s, kQ6Padded);
        CK(cudaGetLastError());
        CK(cudaMemcpyAsync(Y + o0, dy + o0, sizeof(float) * (o1 - o0), cudaMemcpyDeviceToHost, s));
    } else {
        launch_gemm_dense(code, dw, dx, T, n_out, n_in, dy, s, kQ6Padded);
        CK(cudaGetLastError());
        CK(cudaMemcpyAsync(Y, dy, sizeof(float) * (size_t)T * n_out, cudaMemcpyDeviceToHost, s));
    }
    CK(cudaStreamSynchronize(s));
    return 0;
}

int m5_gemv(int code, const float* x, const uint8_t* W, int n_out, int n_in, float* y) {
    std::lock_guard<std::mutex> lk(g_mu);
    const int rc = gemm_impl(code, x, W, 1, n_out, n_in, y, 0, n_out);
    return rc == 0 ? 0 : -1;
}

int m5_gemv_range(int code, const float* x, const uint8_t* W, int n_out, int n_in, float* y, int o0, int o1) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (o0 < 0 || o1 > n_out) return -1;
    const int rc = gemm_impl(code, x, W, 1, n_out, n_in, y, o0, o1);
    return rc == 0 ? 0 : -1;
}

int m5_gemm(int code, const float* X, const uint8_t* W, int T, int n_out, int n_in, float* Y, float* wbuf) {
    (void)wbuf;
    std::lock_guard<std::mutex> lk(g_mu);
    const int rc = gemm_impl(code, X, W, T, n_out, n_in, Y, 0, n_out);
    if (rc) fprintf(stderr, "[draco_moe_b200] m5_gemm: %s\n", g_err.c_str());
    return 0;   // the reference's m5_gemm skips rows it cannot decode and returns 0
}

int m5_gemm_auto(int code, const float* X, const uint8_t* W, int c, int n_out, int n_in, float* Y) {
    if (!code_supported(code)) return -1;
    std::lock_guard<std::mutex> lk(g_mu);
    return gemm_impl(code, X, W, c, n_out, n_in, Y, 0, n_out) == 0 ? 0 : -1;
}

#define DRACO_FUSED(FN, CODE)                                                                  \
    void FN(const float* X, const uint8_t* W, int c, int n_out, int n_in, float* Y) {          \
        std::lock_guard<std::mutex> lk(g_mu);                                                  \
        if (gemm_impl(CODE, X, W, c, n_out, n_in, Y, 0, n_out))                                \
            fail_void(#FN, Y, (size_t)(c > 0 && n_out > 0 ? (size_t)c * n_out : 0));            \
    }
DRACO_FUSED(m5_gemm_q80, DRACO_CODE_Q8_0)
DRACO_FUSED(m5_gemm_q6k, DRACO_CODE_Q6_K)
DRACO_FUSED(m5_gemm_q4k, DRACO_CODE_Q4_K)

int m5_dequant_row(int code, const uint8_t* row, int n_in, float* out) {
    if (!code_supported(code) || n_in % block_values(code) || (code != DRACO_CODE_Q8_0 && n_in % 256)) return -1;
    std::lock_guard<std::mutex> lk(g_mu);
    Ctx* c = get_ctx();
    if (!c) return -1;
    const size_t rb = row_bytes(code, n_in);
    Carver cv;
    const size_t o_w = cv.take<uint8_t>(rb), o_o = cv.take<float>(n_in);
    if (ensure_ws(c, cv.off)) return -1;
    cudaStream_t s = c->stream;
    if (cudaMemcpyAsync(c->ws + o_w, row, rb, cudaMemcpyHostToDevice, s) != cudaSuccess) return -1;
    launch_dequant(code, (const uint8_t*)(c->ws + o_w), 1, n_in, (float*)(c->ws + o_o), s, kQ6File);
    if (cudaMemcpyAsync(out, c->ws + o_o, sizeof(float) * n_in, cudaMemcpyDeviceToHost, s) != cudaSuccess) return -1;
    return cudaStreamSynchronize(s) == cudaSuccess ? 0 : -1;
}

int m6_init_dl(const char* p012, const char* p3, const char* p4, const char* p56, const char* ps) {
    (void)p012, (void)p3, (void)p4, (void)p56, (void)ps;
    const char* mv = getenv("MOE_CHUNK");
    if (mv) g_moe_chunk = atoi(mv);
    return 0;
}

int m6_set_moe_chunk(int v) {
    const int o = g_moe_chunk;
    g_moe_chunk = v;
    return o;
}

void m6_prof_reset(void) {
    for (int i = 0; i < 24; i++) {
        m6_prof_t[i] = 0;
        m6_prof_n[i] = 0;
    }
}
double m6_prof_get(int i) { return (i >= 0 && i < 24) ? m6_prof_t[i] : 0.0; }
long m6_prof_cnt(int i) { return (i >= 0 && i < 24) ? m6_prof_n[i] : 0; }

size_t m6_rowbytes(int code, int n_in) {
    switch (code) {
        case 0: return (size_t)(n_in / 32) * 34;
        case 1: return (size_t)(n_in / 32) * 18;
        case 2: return (size_t)(n_in / 256) * 110;
        case 3: return (size_t)(n_in / 256) * 176;
        case 4: return (size_t)(n_in / 256) * 210;
        case 5: return (size_t)(n_in / 256) * 144;
        case 6: return (size_t)(n_in / 256) * 136;
        case 7: return (size_t)n_in * 2;
        case 8: return (size_t)(n_in / 32) * 22;
        case 9: return (size_t)n_in * 4;
        default: return 0;
    }
}

// ===================================== Part 2 ==========================================

const char* draco_b200_last_error(void) { return g_err.c_str(); }
const char* draco_b200_version(void) { return "draco_moe_b200/0.1 sm_100a"; }

int draco_b200_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

int draco_b200_moe_forward(const DracoMoeLayer* L, const float* X, int T, float* out, int* order_out,
                           float* wtop_out, void* stream) {
    std::lock_guard<std::mutex> lk(g_mu);
    const uint64_t sh3[3] = {(uint64_t)(uintptr_t)L->sh_gate, (uint64_t)(uintptr_t)L->sh_up,
                             (uint64_t)(uintptr_t)L->sh_down};
    const int shc3[3] = {L->sh_code_g, L->sh_code_u, L->sh_code_d};
    const bool has_sh = L->sh_gate && L->sh_up && L->sh_down && L->sh_ff > 0;
    return layer_call(X, T, L->exp_ptrs, L->exp_codes, L->gate_inp, L->probs_b, L->scoring, L->n_exp, L->n_used,
                      L->n_group, L->n_group_used, L->norm_w, L->w_scale, L->inter, L->n_in, L->n_out,
                      has_sh ? sh3 : nullptr, shc3, has_sh ? L->sh_ff : 0, out, order_out, wtop_out,
                      (cudaStream_t)stream);
}

int draco_b200_experts_forward(const DracoMoeLayer* L, const void* X, int T, const int* order, const float* wtop,
                               int ld, int first_expert, float* out, int with_shared, int x_fp16, void* stream) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (order && (!wtop || (ld != 0 && ld < L->n_used) || first_expert < 0)) {
        set_err("draco_b200_experts_forward: wtop missing, ld < n_used or first_expert < 0");
        return -1;
    }
    GivenRoute gr;
    gr.order = order;
    gr.wtop = wtop;
    gr.ld = ld ? ld : L->n_used;
    gr.e_base = first_expert;
    gr.x_half = x_fp16 != 0;
    const uint64_t sh3[3] = {(uint64_t)(uintptr_t)L->sh_gate, (uint64_t)(uintptr_t)L->sh_up,
                             (uint64_t)(uintptr_t)L->sh_down};
    const int shc3[3] = {L->sh_code_g, L->sh_code_u, L->sh_code_d};
    const bool has_sh = with_shared && L->sh_gate && L->sh_up && L->sh_down && L->sh_ff > 0;
    return layer_call(static_cast<const float*>(X), T, L->exp_ptrs, L->exp_codes, L->gate_inp, L->probs_b,
                      L->scoring, L->n_exp, L->n_used, L->n_group, L->n_group_used, L->norm_w, L->w_scale, L->inter,
                      L->n_in, L->n_out, has_sh ? sh3 : nullptr, shc3, has_sh ? L->sh_ff : 0, out, nullptr, nullptr,
                      (cudaStream_t)stream, &gr);
}

int draco_b200_experts_forward_to_ranks(const DracoMoeLayer* L, const void* X, int T, const int* order,
                                        const float* wtop, int ld, int first_expert, float* const* out_blocks,
                                        int block, int x_fp16, void* stream) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!order || !wtop || !out_blocks || !X || ld < L->n_used || first_expert < 0 || block < 1 || L->n_out % 4 ||
        L->n_used > 64) {
        set_err("draco_b200_experts_forward_to_ranks: need order, wtop, out_blocks, ld >= n_used, first_expert >= 0, "
                "block >= 1, n_out %% 4 == 0, n_used <= 64");
        return -1;
    }
    if (!dev_kind(X) || !dev_kind(order) || !dev_kind(wtop) || !dev_kind(out_blocks)) {
        set_err("draco_b200_experts_forward_to_ranks: device pointers only");
        return -1;
    }
    GivenRoute gr;
    gr.order = order;
    gr.wtop = wtop;
    gr.ld = ld;
    gr.e_base = first_expert;
    gr.x_half = x_fp16 != 0;
    gr.out_blk = out_blocks;
    gr.out_block = block;
    return layer_call(static_cast<const float*>(X), T, L->exp_ptrs, L->exp_codes, L->gate_inp, L->probs_b,
                      L->scoring, L->n_exp, L->n_used, L->n_group, L->n_group_used, L->norm_w, L->w_scale, L->inter,
                      L->n_in, L->n_out, nullptr, nullptr, 0, nullptr, nullptr, nullptr, (cudaStream_t)stream, &gr);
}

int draco_b200_route(const DracoMoeLayer* L, const float* X, int T, int* order, float* wtop, void* stream) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (int rc = validate_shape(L->n_exp, L->n_used, L->inter, L->n_in, L->n_out, L->scoring ? L->n_group : 1,
                                L->n_group_used))
        return rc;
    if (T <= 0) return 0;
    Ctx* c = get_ctx();
    if (!c) return -3;
    const float* d_gi = (const float*)dev_range(c, L->gate_inp, sizeof(float) * (size_t)L->n_exp * L->n_in);
    if (!d_gi) return -1;
    RouterParams rp{L->scoring, L->n_exp, L->n_used, L->n_in, L->scoring ? L->n_group : 1, L->n_group_used,
                    L->norm_w, L->w_scale, nullptr};
    if (L->scoring && L->probs_b) {
        rp.probs_b = (const float*)dev_range(c, L->probs_b, sizeof(float) * L->n_exp);
        if (!rp.probs_b) return -1;
    }
    const size_t n = (size_t)T * L->n_used;
    Carver cv;
    const size_t o_x = cv.take<float>((size_t)T * L->n_in), o_lg = cv.take<float>((size_t)T * L->n_exp);
    const size_t o_o = cv.take<int>(n), o_w = cv.take<float>(n), o_e = cv.take<int>(1);
    if (int rc = ensure_ws(c, cv.off)) return rc;
    RouteBufs b{};
    b.logits = (float*)(c->ws + o_lg);
    b.order = (int*)(c->ws + o_o);
    b.wtop = (float*)(c->ws + o_w);
    b.err = (int*)(c->ws + o_e);
    const bool dev_io = dev_kind(X);
    cudaStream_t s = (dev_io && stream) ? (cudaStream_t)stream : c->stream;
    if (dev_io && !stream)
        if (int rc = after_legacy_stream(c)) return rc;
    const float* dx = X;
    if (!dev_io) {
        CK(cudaMemcpyAsync(c->ws + o_x, X, sizeof(float) * (size_t)T * L->n_in, cudaMemcpyHostToDevice, s));
        dx = (const float*)(c->ws + o_x);
    }
    CK(cudaMemsetAsync(b.err, 0, sizeof(int), s));
    launch_router_logits(dx, d_gi, T, L->n_exp, L->n_in, b.logits, s);
    launch_router_select(rp, T, b, s);
    g_launches += 2;
    CK(cudaGetLastError());
    const cudaMemcpyKind k = dev_io ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost;
    CK(cudaMemcpyAsync(order, b.order, sizeof(int) * n, k, s));
    CK(cudaMemcpyAsync(wtop, b.wtop, sizeof(float) * n, k, s));
    if (dev_io && stream) return 0;
    int h_err = 0;
    CK(cudaMemcpyAsync(&h_err, b.err, sizeof(int), cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    if (h_err) {
        set_err("routing found fewer eligible experts than n_used, code %d", h_err);
        return -2;
    }
    return 0;
}

int draco_b200_profile(int enable) {
    std::lock_guard<std::mutex> lk(g_mu);
    resolve_prof();
    const int o = g_prof ? 1 : 0;
    g_prof = enable != 0;
    for (int i = 0; i < kPhases; i++) {
        g_phase_ms[i] = 0;
        g_phase_n[i] = 0;
    }
    return o;
}

int draco_b200_profile_read(double* ms, long* counts, int n) {
    std::lock_guard<std::mutex> lk(g_mu);
    resolve_prof();
    for (int i = 0; i < n && i < kPhases; i++) {
        if (ms) ms[i] = g_phase_ms[i];
        if (counts) counts[i] = g_phase_n[i];
    }
    return kPhases;
}

// ---- expert-parallel exchange kernels (device pointers, asynchronous on the given stream) ----
static bool ep_ptrs_ok(std::initializer_list<const void*> ps, const char* who) {
    for (const void* p : ps) {
        if (p && (!dev_kind(p) || ((uintptr_t)p & 15))) {
            set_err("%s: buffers must be 16-byte aligned device memory", who);
            return false;
        }
    }
    return true;
}

int draco_b200_ep_plan(const int* order, int T, int K, int n_exp, int n_ranks, int block, int* counts, int* row_of,
                       int* src_tok, void* stream) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (n_ranks < 1 || n_ranks > kEpMaxRanks || n_exp % n_ranks || K < 1 || T < 0 || (block && block < T) ||
        block < 0) {
        set_err("draco_b200_ep_plan: need 1 <= n_ranks <= %d dividing n_exp, K >= 1, block 0 or >= T", kEpMaxRanks);
        return -1;
    }
    if (!order || !counts || !row_of || !src_tok) {
        set_err("draco_b200_ep_plan: null pointer");
        return -1;
    }
    if (!ep_ptrs_ok({order, counts, row_of, src_tok}, "draco_b200_ep_plan")) return -1;
    launch_ep_plan(order, T, K, n_exp, n_ranks, block, counts, row_of, src_tok, (cudaStream_t)stream);
    g_launches += 1;
    CK(cudaGetLastError());
    return 0;
}

int draco_b200_ep_pack(const float* X, const int* order, const float* wtop, const int* counts, int n_ranks,
                       const int* src_tok, int block, int cap, int K, int H, float* send_x, int* send_meta,
                       void* stream) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (n_ranks < 1 || n_ranks > kEpMaxRanks || H % 4 || K < 1 || cap < 0 || block < 0) {
        set_err("draco_b200_ep_pack: need 1 <= n_ranks <= %d, H %% 4 == 0, K >= 1", kEpMaxRanks);
        return -1;
    }
    if (!ep_ptrs_ok({X, order, wtop, counts, src_tok, send_x, send_meta}, "draco_b200_ep_pack")) return -1;
    if (cap == 0) return 0;
    launch_ep_pack(X, order, wtop, counts, n_ranks, src_tok, block, cap, K, H, send_x, send_meta,
                   (cudaStream_t)stream);
    g_launches += 1;
    CK(cudaGetLastError());
    return 0;
}

int draco_b200_ep_combine(const float* back, const int* row_of, int T, int n_ranks, int H, const float* shared,
                          float* out, void* stream) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (n_ranks < 1 || n_ranks > kEpMaxRanks || H % 4 || T < 0) {
        set_err("draco_b200_ep_combine: need 1 <= n_ranks <= %d, H %% 4 == 0", kEpMaxRanks);
        return -1;
    }
    if (T == 0) return 0;
    if (!back || !row_of || !out) {
        set_err("draco_b200_ep_combine: null pointer");
        return -1;
    }
    if (!ep_ptrs_ok({back, row_of, shared, out}, "draco_b200_ep_combine")) return -1;
    launch_ep_combine(back, row_of, T, n_ranks, H, shared, out, (cudaStream_t)stream);
    g_launches += 1;
    CK(cudaGetLastError());
    return 0;
}

// ---- peer memory for the expert-parallel exchange (CUDA IPC; one process per GPU) ----
int draco_b200_ep_mem_alloc(size_t bytes, void** ptr, void* handle) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!ptr || !handle || bytes == 0) {
        set_err("draco_b200_ep_mem_alloc: null output or zero size");
        return -1;
    }
    *ptr = nullptr;
    void* p = nullptr;
    CK(cudaMalloc(&p, bytes));
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaMemset(p, 0, bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        set_err("draco_b200_ep_mem_alloc: %s", cudaGetErrorString(e));
        return -3;
    }
    memcpy(handle, &h, sizeof h);
    *ptr = p;
    return 0;
}

int draco_b200_ep_mem_open(const void* handle, void** ptr) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!ptr || !handle) {
        set_err("draco_b200_ep_mem_open: null argument");
        return -1;
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof h);
    CK(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
    return 0;
}

int draco_b200_ep_mem_close(void* ptr) {
    std::lock_guard<std::mutex> lk(g_mu);
    CK(cudaDeviceSynchronize());
    CK(cudaIpcCloseMemHandle(ptr));
    return 0;
}

int draco_b200_ep_mem_free(void* ptr) {
    std::lock_guard<std::mutex> lk(g_mu);
    CK(cudaDeviceSynchronize());
    CK(cudaFree(ptr));
    return 0;
}

int draco_b200_ep_push(const float* X, const int* order, const float* wtop, const int* counts, int n_ranks, int rank,
                       const int* src_tok, int block, int K, int H, void* const* dst_x, int x_fp16,
                       int* const* dst_meta, void* stream) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (n_ranks < 1 || n_ranks > kEpMaxRanks || rank < 0 || rank >= n_ranks || H % (x_fp16 ? 8 : 4) || K < 1 ||
        block < 1) {
        set_err("draco_b200_ep_push: need 0 <= rank < n_ranks <= %d, H %% 4 == 0, K >= 1, block >= 1", kEpMaxRanks);
        return -1;
    }
    if (!X || !order || !wtop || !counts || !src_tok || !dst_x || !dst_meta) {
        set_err("draco_b200_ep_push: null pointer");
        return -1;
    }
    if (!ep_ptrs_ok({X, order, wtop, counts, src_tok, dst_x, dst_meta}, "draco_b200_ep_push")) return -1;
    launch_ep_push(X, order, wtop, counts, n_ranks, rank, src_tok, block, K, H, dst_x, x_fp16 != 0, dst_meta,
                   (cudaStream_t)stream);
    g_launches += 1;
    CK(cudaGetLastError());
    return 0;
}

int draco_b200_ep_barrier(unsigned* const* peer_flags, unsigned* my_flags, unsigned* epoch, int n_ranks, int rank,
                          int* status, void* stream) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (n_ranks < 1 || n_ranks > kEpMaxRanks || rank < 0 || rank >= n_ranks) {
        set_err("draco_b200_ep_barrier: need 0 <= rank < n_ranks <= %d", kEpMaxRanks);
        return -1;
    }
    if (!peer_flags || !my_flags || !epoch || !status) {
        set_err("draco_b200_ep_barrier: null pointer");
        return -1;
    }
    if (!ep_ptrs_ok({peer_flags, my_flags, epoch, status}, "draco_b200_ep_barrier")) return -1;
    launch_ep_barrier(peer_flags, my_flags, epoch, n_ranks, rank, status, (cudaStream_t)stream);
    g_launches += 1;
    CK(cudaGetLastError());
    return 0;
}

int draco_b200_ep_pull_combine(const float* const* src_partial, const int* row_of, int T, int n_ranks, int rank,
                               int block, int H, const float* shared, float* out, void* stream) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (n_ranks < 1 || n_ranks > kEpMaxRanks || rank < 0 || rank >= n_ranks || H % 4 || T < 0 || block < T) {
        set_err("draco_b200_ep_pull_combine: need 0 <= rank < n_ranks <= %d, H %% 4 == 0, T <= block", kEpMaxRanks);
        return -1;
    }
    if (T == 0) return 0;
    if (!src_partial || !row_of || !out) {
        set_err("draco_b200_ep_pull_combine: null pointer");
        return -1;
    }
    if (!ep_ptrs_ok({src_partial, row_of, shared, out}, "draco_b200_ep_pull_combine")) return -1;
    launch_ep_pull_combine(src_partial, row_of, T, n_ranks, rank, block, H, shared, out, (cudaStream_t)stream);
    g_launches += 1;
    CK(cudaGetLastError());
    return 0;
}

long draco_b200_launch_count(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    return g_launches;
}

int draco_b200_set_gemm_path(int mode) {
    std::lock_guard<std::mutex> lk(g_mu);
    const int o = gemm_path();
    if (mode >= 0 && mode <= 2) g_gemm_path = mode;
    return o;
}

int draco_b200_set_fused_decode(int on) {
    std::lock_guard<std::mutex> lk(g_mu);
    const int o = fused_decode_enabled() ? 1 : 0;
    if (on == 0 || on == 1) {
        g_fused_decode = on;
        if (Ctx* c = get_ctx()) drop_graphs(c);   // captured calls hold the previous choice
    }
    return o;
}

int draco_b200_test_fused_barrier_extra(int n) {
    std::lock_guard<std::mutex> lk(g_mu);
    const int o = g_fd_extra;
    if (n >= 0) {
        g_fd_extra = n;
        if (Ctx* c = get_ctx()) drop_graphs(c);
    }
    return o;
}

int draco_b200_set_act_mode(int mode) {
    std::lock_guard<std::mutex> lk(g_mu);
    const int o = g_act_mode;
    if (mode == 0 || mode == 1) g_act_mode = mode;
    return o;
}

int draco_b200_register(const void* host, size_t bytes) {
    std::lock_guard<std::mutex> lk(g_mu);
    Ctx* c = get_ctx();
    if (!c) return -3;
    return dev_range(c, host, bytes) ? 0 : -1;
}

int draco_b200_forget(const void* host) {
    std::lock_guard<std::mutex> lk(g_mu);
    Ctx* c = get_ctx();
    if (!c) return -3;
    auto it = c->regions.find((uintptr_t)host);
    if (it == c->regions.end()) return -1;
    drop_region(c, it);
    return 0;
}

void draco_b200_reset(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    Ctx* c = get_ctx();
    if (!c) return;
    cudaDeviceSynchronize();   // asynchronous calls on any stream are done with the buffers
    drop_tables(c);            // tables, their tensor maps and the captured graphs
    for (auto& kv : c->regions) cudaFree(kv.second.dev);
    c->regions.clear();
    c->reg_bytes = 0;
    if (c->ws) cudaFree(c->ws);
    for (char* w : c->ws_retired) cudaFree(w);
    c->ws_retired.clear();
    c->ws = nullptr;
    c->ws_cap = 0;
    c->ws_captured = false;
    c->ws_event_set = false;
}

size_t draco_b200_registered_bytes(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    Ctx* c = get_ctx();
    return c ? c->reg_bytes : 0;
}

// ---- test hooks: host arrays in, host arrays out ----
int draco_b200_expf(const float* x, float* y, long n) {
    std::lock_guard<std::mutex> lk(g_mu);
    Ctx* c = get_ctx();
    if (!c) return -3;
    Carver cv;
    const size_t o_x = cv.take<float>(n), o_y = cv.take<float>(n);
    if (int rc = ensure_ws(c, cv.off)) return rc;
    cudaStream_t s = c->stream;
    if (int rc = stage_in(c, s, o_x, x, n)) return rc;
    launch_expf((const float*)(c->ws + o_x), (float*)(c->ws + o_y), n, s);
    CK(cudaGetLastError());
    CK(cudaMemcpyAsync(y, c->ws + o_y, sizeof(float) * n, cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    return 0;
}

int draco_b200_router_logits(const float* X, const float* W, int T, int E, int H, float* logits) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (T <= 0 || E <= 0 || H <= 0) return -1;
    Ctx* c = get_ctx();
    if (!c) return -3;
    Carver cv;
    const size_t o_x = cv.take<float>((size_t)T * H), o_w = cv.take<float>((size_t)E * H);
    const size_t o_l = cv.take<float>((size_t)T * E);
    if (int rc = ensure_ws(c, cv.off)) return rc;
    cudaStream_t s = c->stream;
    if (int rc = stage_in(c, s, o_x, X, (size_t)T * H)) return rc;
    if (int rc = stage_in(c, s, o_w, W, (size_t)E * H)) return rc;
    launch_router_logits((const float*)(c->ws + o_x), (const float*)(c->ws + o_w), T, E, H, (float*)(c->ws + o_l), s);
    CK(cudaGetLastError());
    CK(cudaMemcpyAsync(logits, c->ws + o_l, sizeof(float) * T * E, cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    return 0;
}

int draco_b200_q8k_quantize(const float* x, int n, float* d, int8_t* q, int16_t* bsums) {
    if (n % 256) return -1;
    std::lock_guard<std::mutex> lk(g_mu);
    Ctx* c = get_ctx();
    if (!c) return -3;
    const int nb = n / 256;
    Carver cv;
    const size_t o_x = cv.take<float>(n), o_d = cv.take<float>(nb), o_q = cv.take<int8_t>(n);
    const size_t o_b = cv.take<int16_t>((size_t)nb * 16);
    if (int rc = ensure_ws(c, cv.off)) return rc;
    cudaStream_t s = c->stream;
    if (int rc = stage_in(c, s, o_x, x, n)) return rc;
    launch_q8k_quantize((const float*)(c->ws + o_x), 1, n, (float*)(c->ws + o_d), (int8_t*)(c->ws + o_q),
                        (int16_t*)(c->ws + o_b), s);
    CK(cudaGetLastError());
    CK(cudaMemcpyAsync(d, c->ws + o_d, sizeof(float) * nb, cudaMemcpyDeviceToHost, s));
    CK(cudaMemcpyAsync(q, c->ws + o_q, n, cudaMemcpyDeviceToHost, s));
    CK(cudaMemcpyAsync(bsums, c->ws + o_b, sizeof(int16_t) * nb * 16, cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    return 0;
}

int draco_b200_q8k_block_dots(int code, const uint8_t* W, int rows, int n_in, const int8_t* q, const int16_t* bsums,
                              int32_t* out2) {
    if ((code != DRACO_CODE_Q4_K && code != DRACO_CODE_Q6_K) || n_in % 256) return -1;
    std::lock_guard<std::mutex> lk(g_mu);
    Ctx* c = get_ctx();
    if (!c) return -3;
    const int nb = n_in / 256;
    const size_t wb = (size_t)rows * row_bytes(code, n_in);
    Carver cv;
    const size_t o_w = cv.take<uint8_t>(wb), o_q = cv.take<int8_t>(n_in), o_b = cv.take<int16_t>((size_t)nb * 16);
    const size_t o_o = cv.take<int32_t>((size_t)rows * nb * 2);
    if (int rc = ensure_ws(c, cv.off)) return rc;
    cudaStream_t s = c->stream;
    if (int rc = stage_in(c, s, o_w, W, wb)) return rc;
    if (int rc = stage_in(c, s, o_q, q, n_in)) return rc;
    if (int rc = stage_in(c, s, o_b, bsums, (size_t)nb * 16)) return rc;
    launch_q8k_block_dots(code, (const uint8_t*)(c->ws + o_w), rows, n_in, (const int8_t*)(c->ws + o_q),
                          (const int16_t*)(c->ws + o_b), (int32_t*)(c->ws + o_o), s, kQ6File);
    CK(cudaGetLastError());
    CK(cudaMemcpyAsync(out2, c->ws + o_o, sizeof(int32_t) * rows * nb * 2, cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    return 0;
}

int draco_b200_gemv_q8k(int code, const uint8_t* W, int rows, int n_in, const int8_t* q, const float* d,
                        const int16_t* bsums, float* y) {
    if ((code != DRACO_CODE_Q4_K && code != DRACO_CODE_Q6_K) || n_in % 256) return -1;
    std::lock_guard<std::mutex> lk(g_mu);
    Ctx* c = get_ctx();
    if (!c) return -3;
    const int nb = n_in / 256;
    const size_t wb = (size_t)rows * row_bytes(code, n_in);
    Carver cv;
    const size_t o_w = cv.take<uint8_t>(wb), o_q = cv.take<int8_t>(n_in), o_b = cv.take<int16_t>((size_t)nb * 16);
    const size_t o_d = cv.take<float>(nb), o_y = cv.take<float>(rows);
    if (int rc = ensure_ws(c, cv.off)) return rc;
    cudaStream_t s = c->stream;
    if (int rc = stage_in(c, s, o_w, W, wb)) return rc;
    if (int rc = stage_in(c, s, o_q, q, n_in)) return rc;
    if (int rc = stage_in(c, s, o_b, bsums, (size_t)nb * 16)) return rc;
    if (int rc = stage_in(c, s, o_d, d, nb)) return rc;
    launch_gemv_q8k(code, (const uint8_t*)(c->ws + o_w), rows, n_in, (const int8_t*)(c->ws + o_q),
                    (const float*)(c->ws + o_d), (const int16_t*)(c->ws + o_b), (float*)(c->ws + o_y), s, kQ6File);
    CK(cudaGetLastError());
    CK(cudaMemcpyAsync(y, c->ws + o_y, sizeof(float) * rows, cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    return 0;
}

}  // extern "C"
