// Allocation-free variant of the chunked-prefill MoE op (m6_moe_tok semantics) for callers
// that cannot let a library allocate device memory: an engine that reserves HBM for its
// weights and KV cache up front and treats any allocation outside its pool as a budget
// violation, or a per-token loop where cudaMalloc's implicit device synchronisation would
// stall the pipeline.
//
// The op's scratch (expert pointer table, dispatch lists, intermediate activations) lives in
// one file-scope device array of fixed size, kNoAllocScratchBytes.  Every GPU that loads this
// library holds that array until the process exits.  All calls share it and it keeps the
// previous call's contents; everything that must start at zero is cleared by the call itself.
// Two calls whose work overlaps on the GPU (different streams, or different host threads on
// one device) race on the array: serialise them.
//
// The first call on a device looks up the array's device address (cudaGetSymbolAddress) with
// that device current and remembers it.
// Nothing here calls cudaMalloc, cudaFree or any other allocating routine.
#include "../../include/draco_moe_b200.h"
#include "kernels.cuh"

#include <cstdio>
#include <mutex>

using namespace draco;

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;   // 32 MiB per device

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// per-device address of g_noalloc_scratch (host code cannot use the symbol as an address)
unsigned char* g_scratch_addr[64];
std::mutex g_noalloc_mu;

size_t up256(size_t v) { return (v + 255) & ~size_t(255); }

bool codes_ok(int c) { return c == DRACO_CODE_Q4_K || c == DRACO_CODE_Q6_K || c == DRACO_CODE_Q8_0; }

// errors go to stderr (no host allocation on any path) and come back as the return code
int fail(int rc, const char* msg, const char* detail = "") {
    fprintf(stderr, "[draco_moe_b200] draco_b200_moe_tok_noalloc: %s%s\n", msg, detail);
    return rc;
}

// scratch bytes one call needs (the layout carved below)
size_t scratch_bytes(int T, int n_used, int inter, int n_out, int n_exp) {
    const size_t n = (size_t)(T > 0 ? T : 0) * (size_t)(n_used > 0 ? n_used : 0);
    size_t off = 0;
    off += up256(sizeof(uint64_t) * 3 * (size_t)n_exp);      // device copy of the pointer table
    off += up256(sizeof(int) * (size_t)n_exp);               // counts
    off += up256(sizeof(int) * ((size_t)n_exp + 1));         // off
    off += up256(sizeof(int) * (n ? n : 1));                 // ilist
    off += up256(sizeof(int) * (n ? n : 1));                 // pos_of
    off += up256(sizeof(int) * (size_t)n_exp);               // active
    off += up256(sizeof(int));                               // n_active
    off += up256(sizeof(int) * dispatch_chunk_ints((int)n, n_exp));   // dispatch chunk counts
    off += up256(sizeof(float) * (n ? n : 1) * (size_t)inter);   // act
    off += up256(sizeof(float) * (n ? n : 1) * (size_t)n_out);   // y
    return off;
}

}  // namespace

extern "C" int draco_b200_moe_tok_noalloc(const float* X, const int* order, const float* wtop,
                                          const uint64_t* ep_dev, const int* ec, int T, int n_used,
                                          int inter, int n_in, int n_out, int n_exp, float* out,
                                          void* stream) {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (T == 0) return 0;
    if (T < 0 || n_exp <= 0 || n_exp > 512 || n_used <= 0 || n_used > 64 || n_used > n_exp || inter <= 0 ||
        n_in <= 0 || n_out <= 0)
        return fail(-1, "unsupported shape");
    if (!X || !order || !wtop || !ep_dev || !ec || !out) return fail(-1, "null argument");
    if (((uintptr_t)X & 15) || ((uintptr_t)out & 15)) return fail(-1, "X and out must be 16-byte aligned");
    const int cg = ec[0], cu = ec[1], cd = ec[2];
    for (int e = 0; e < n_exp; e++)
        if (ec[3 * e] != cg || ec[3 * e + 1] != cu || ec[3 * e + 2] != cd)
            return fail(-1, "experts must share their formats");
    if (!codes_ok(cg) || !codes_ok(cu) || !codes_ok(cd)) return fail(-1, "unsupported weight format code");
    if (n_in % block_values(cg) || n_in % block_values(cu) || inter % block_values(cd) ||
        (cg != DRACO_CODE_Q8_0 && n_in % 256) || (cu != DRACO_CODE_Q8_0 && n_in % 256) ||
        (cd != DRACO_CODE_Q8_0 && inter % 256))
        return fail(-1, "row length not a multiple of the block size");
    // the row decoders read Q4_K superblocks with 4-byte loads from 16-byte aligned blocks and
    // Q6_K / Q8_0 blocks with 2-byte loads: a misaligned table entry is refused here, before
    // anything runs, instead of faulting on the device
    for (int e = 0; e < n_exp; e++)
        for (int k = 0; k < 3; k++) {
            const uint64_t a = ep_dev[3 * e + k];
            const uint64_t align = ec[3 * e + k] == DRACO_CODE_Q4_K ? 16 : 2;
            if (a == 0 || a % align) return fail(-1, "weight address null or misaligned for its format");
        }
    const size_t need = scratch_bytes(T, n_used, inter, n_out, n_exp);
    if (need > kNoAllocScratchBytes) {
        fprintf(stderr,
                "[draco_moe_b200] draco_b200_moe_tok_noalloc: this call needs %zu scratch bytes, more than the "
                "fixed maximum of %zu; pass fewer tokens per call\n", need, kNoAllocScratchBytes);
        return -4;
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        return fail(-3, "no CUDA device");
    }
    if (!g_scratch_addr[dev]) {
        // set-up, once per device, with that device current
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) return fail(-3, "cudaGetSymbolAddress failed: ", cudaGetErrorString(e));
        g_scratch_addr[dev] = (unsigned char*)p;
    }
    unsigned char* base = g_scratch_addr[dev];
    cudaStream_t s = (cudaStream_t)stream;
    const size_t n = (size_t)T * n_used;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        unsigned char* p = base + off;
        off += up256(bytes);
        return p;
    };
    uint64_t* d_ptrs = (uint64_t*)take(sizeof(uint64_t) * 3 * (size_t)n_exp);
    RouteBufs rb{};
    rb.counts = (int*)take(sizeof(int) * n_exp);
    rb.off = (int*)take(sizeof(int) * (n_exp + 1));
    rb.ilist = (int*)take(sizeof(int) * n);
    rb.pos_of = (int*)take(sizeof(int) * n);
    rb.active = (int*)take(sizeof(int) * n_exp);
    rb.n_active = (int*)take(sizeof(int));
    rb.chunk_counts = (int*)take(sizeof(int) * dispatch_chunk_ints((int)n, n_exp));
    float* act = (float*)take(sizeof(float) * n * inter);
    float* y = (float*)take(sizeof(float) * n * n_out);
    rb.order = const_cast<int*>(order);
    rb.wtop = const_cast<float*>(wtop);
    // the pointer table goes into the scratch array; the dispatch clears its own counters
    if (cudaMemcpyAsync(d_ptrs, ep_dev, sizeof(uint64_t) * 3 * (size_t)n_exp, cudaMemcpyHostToDevice, s) !=
        cudaSuccess)
        return fail(-3, "pointer table copy failed");
    launch_dispatch(T, n_used, n_exp, rb, s);
    ExpertTable et{(const uint8_t* const*)d_ptrs};
    const int na_max = n_exp < T * n_used ? n_exp : T * n_used;
    launch_gateup_codes(et, cg, cu, rb.active, rb.n_active, na_max, rb.off, rb.ilist, n_used, X, inter, n_in, act,
                        s, kQ6File);
    launch_down_code(et, cd, rb.active, rb.n_active, na_max, rb.off, act, inter, n_out, y, s, kQ6File);
    launch_combine(y, order, wtop, rb.pos_of, T, n_used, n_exp, n_out, nullptr, out, s);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(-3, "launch failed: ", cudaGetErrorString(e));
    return 0;
}
