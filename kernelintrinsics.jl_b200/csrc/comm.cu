// comm.cu -- communicators and the range-sharded reduce / scan / compaction over several GPUs.
//
// The reference's multi-device surface is device enumeration and selection (src/device.jl:1-19,
// ext/CUDA/device.jl:4-13) plus the System scope of @access / @fence
// (ext/CUDA/scopes_ordering.jl:13); the sharded operations are built from those pieces here.
//
// Each rank owns a contiguous shard.  The only data that crosses NVLink is one 8-byte value per rank
// and operation (a Float64 partial sum, an Int64 shard total, a UInt64 count), exchanged by the
// exchange kernel below over peer memory:
//
//   every rank has a 2 KiB exchange buffer of slots {value, epoch}, [2 parities][64 writers];
//   a call takes epoch e = (device epoch counter) + 1;  lane q of the exchange kernel stores this
//   rank's value into slot [e & 1][rank] of rank q's buffer (plain peer stores: st.relaxed.sys of the
//   value, then st.release.sys of the epoch), then waits, with ld.acquire.sys on ITS OWN buffer, until
//   slot [e & 1][q] carries epoch e (a bounded wait: %globaltimer against the context's limit; on
//   timeout KI_DEV_TIMEOUT is latched and the value taken as 0).  Lane 0 folds the values in rank
//   order (deterministic, the same bits on every rank) and writes the epoch counter back.
//
// Why two parities are enough: every call waits for every rank's value, so rank r can only publish
// epoch e+2 after it has seen epoch e+1 from every rank q, which q publishes only after its own wait
// for epoch e has read r's epoch-e slot.  So a slot is never overwritten before it has been read.
// The waits poll local memory; the only NVLink traffic is the 16-byte stores.
//
// Multi-process communicators (one process per GPU) exchange the buffers' IPC handles with one NCCL
// all-gather at set-up (ncclGetUniqueId / ncclCommInitRankConfig, loaded with dlopen so the library
// does not link NCCL); the data path then needs no NCCL.  When peer mappings cannot be made (no P2P
// between the GPUs) the communicator falls back to an ncclAllGather of the 8-byte values on the
// caller's stream, followed by the same fold.  Single-process communicators (one host thread driving
// several GPUs, ki_comm_create) use peer access (cudaDeviceEnablePeerAccess) and no NCCL at all.
// No cluster multicast, multimem or TMA touches peer memory: the peer accesses are plain 16-byte
// stores.
#include <dlfcn.h>
#include <nccl.h>  // types and NCCL_CONFIG_INITIALIZER only: the functions are looked up with dlsym

#include <chrono>
#include <cstring>
#include <thread>
#include <vector>

#include "ki/common.cuh"
#include "ki/intrinsics.cuh"

// Prepares a scan of up to n elements (scratch, kernel attributes) so that it can be enqueued later
// without a blocking call (scan.cu).
__attribute__((visibility("hidden"))) int ki_scan_i64_reserve(ki_ctx* ctx, size_t n);

namespace {

constexpr int kMaxRanks = KI_COMM_MAX_RANKS;

struct XSlot {
    uint64_t value;
    uint64_t epoch;
};
constexpr size_t kXBufBytes = 2 * kMaxRanks * sizeof(XSlot);  // [parity][writer]

// Local device words of a communicator (uint64 indices).
enum : int {
    W_EPOCH = 0,        // epoch of the last completed exchange
    W_LOCAL = 1,        // this rank's value of the current operation
    W_GATHERED = 8,     // [kMaxRanks] values gathered by NCCL (fallback exchange)
    W_PEERS = W_GATHERED + kMaxRanks,  // [kMaxRanks] exchange buffers as mapped in this process
    W_SEED = W_PEERS + kMaxRanks,      // the sharded scan's seed (sum of lower ranks' totals)
    W_OFFSET = W_SEED + 1,             // compaction offset / total when the caller passes none
    W_TOTAL = W_SEED + 2,
    W_COUNT = W_SEED + 3,
    W_WORDS = W_SEED + 8
};

enum XFold : int {
    XF_SUM_F64 = 0,    // Float64 total of the ranks' partials, in rank order
    XF_PREFIX_I64 = 1, // Int64 (wrapping) sum of the lower ranks' values, and of all
    XF_PREFIX_U64 = 2  // UInt64 sum of the lower ranks' values, and of all
};

struct XArgs {
    XSlot* const* peers;      // peer exchange: every rank's buffer as mapped here (null: NCCL gathered)
    XSlot* mine;              // this rank's buffer
    const uint64_t* gathered; // NCCL fallback: the ranks' values
    const uint64_t* local;    // this rank's value
    uint64_t* epoch;
    int nranks, rank, fold;
    double* out_f64;
    float* out_f32;
    uint64_t* out_prefix;     // sum of lower ranks (Int64 / UInt64)
    uint64_t* out_total;      // sum of all ranks
    uint32_t* status;
    uint64_t timeout_ns;
};

__global__ void __launch_bounds__(32) exchange_kernel(XArgs a) {
    __shared__ uint64_t vals[kMaxRanks];
    // a kernel launched after this one with programmatic stream serialization (the next step's
    // reduce) may be dispatched now; it waits for this kernel to complete before touching memory
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int lane = (int)threadIdx.x;
    const uint64_t v = *a.local;
    uint64_t e = 0;
    if (a.peers) {
        e = *a.epoch + 1;
        const int par = (int)(e & 1);
        for (int q = lane; q < a.nranks; q += 32) {  // publish into every rank's buffer
            XSlot* dst = a.peers[q] + par * kMaxRanks + a.rank;
            ki::store<ki::Order::Relaxed, ki::Scope::System>(&dst->value, v);
            ki::store<ki::Order::Release, ki::Scope::System>(&dst->epoch, e);
        }
        for (int q = lane; q < a.nranks; q += 32) {  // wait for every rank's value in this buffer
            XSlot* src = a.mine + par * kMaxRanks + q;
            uint64_t t0 = 0;
            bool ok = true;
            while (ki::load<ki::Order::Acquire, ki::Scope::System>(&src->epoch) != e) {
                const uint64_t now = ki::globaltimer_ns();
                if (t0 == 0) t0 = now;
                if (now - t0 > a.timeout_ns) {
                    atomicOr(a.status, (uint32_t)KI_DEV_TIMEOUT);
                    ok = false;
                    break;
                }
            }
            vals[q] = ok ? ki::load<ki::Order::Relaxed, ki::Scope::System>(&src->value) : 0;
        }
    } else {
        for (int q = lane; q < a.nranks; q += 32) vals[q] = a.gathered[q];
    }
    __syncwarp();
    if (lane != 0) return;
    if (a.fold == XF_SUM_F64) {
        double t = 0.0;
        for (int q = 0; q < a.nranks; ++q) t += __longlong_as_double((long long)vals[q]);
        if (a.out_f64) *a.out_f64 = t;
        if (a.out_f32) *a.out_f32 = (float)t;
    } else {  // two's-complement sums: the same bits for Int64 (wrapping) and UInt64
        uint64_t below = 0, all = 0;
        for (int q = 0; q < a.nranks; ++q) {
            if (q < a.rank) below += vals[q];
            all += vals[q];
        }
        if (a.out_prefix) *a.out_prefix = below;
        if (a.out_total) *a.out_total = all;
    }
    if (a.peers) *a.epoch = e;
}

// ---- NCCL, looked up at run time ------------------------------------------------------------
struct Nccl {
    bool tried = false, ok = false;
    void* h = nullptr;
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
};
Nccl g_nccl;
std::mutex g_nccl_mutex;

const Nccl* nccl() {
    std::lock_guard<std::mutex> lock(g_nccl_mutex);
    if (g_nccl.tried) return g_nccl.ok ? &g_nccl : nullptr;
    g_nccl.tried = true;
    // an NCCL already in the process (e.g. PyTorch's) is found by its soname first
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
    if (!h) return nullptr;
    g_nccl.h = h;
#define KI_NCCL_SYM(field, name) g_nccl.field = reinterpret_cast<decltype(g_nccl.field)>(dlsym(h, name))
    KI_NCCL_SYM(GetUniqueId, "ncclGetUniqueId");
    KI_NCCL_SYM(CommInitRankConfig, "ncclCommInitRankConfig");
    KI_NCCL_SYM(AllGather, "ncclAllGather");
    KI_NCCL_SYM(CommDestroy, "ncclCommDestroy");
    KI_NCCL_SYM(CommFinalize, "ncclCommFinalize");
    KI_NCCL_SYM(CommAbort, "ncclCommAbort");
    KI_NCCL_SYM(CommGetAsyncError, "ncclCommGetAsyncError");
    KI_NCCL_SYM(GetErrorString, "ncclGetErrorString");
#undef KI_NCCL_SYM
    g_nccl.ok = g_nccl.GetUniqueId && g_nccl.CommInitRankConfig && g_nccl.AllGather && g_nccl.CommDestroy &&
                g_nccl.CommFinalize && g_nccl.CommAbort && g_nccl.CommGetAsyncError && g_nccl.GetErrorString;
    return g_nccl.ok ? &g_nccl : nullptr;
}

// What every rank contributes at set-up (gathered with one ncclAllGather).
struct RankRecord {
    cudaIpcMemHandle_t xbuf;  // this rank's exchange buffer
    char uuid[16];            // the GPU, to refuse two ranks on one GPU
    int32_t ipc_ok;           // filled in a second round: every peer buffer could be mapped
    int32_t pad[11];
};
static_assert(sizeof(RankRecord) == 128, "rank record layout");

}  // namespace

struct ki_comm {
    int nranks = 0, rank = 0, device = 0;
    int exchange = KI_XCHG_PEER;
    bool multi_process = false;
    ki_ctx* ctx = nullptr;         // owned: the sharded kernels' scratch and status word
    ncclComm_t nc = nullptr;       // multi-process only
    cudaStream_t setup = nullptr;  // set-up and tear-down collectives
    XSlot* xbuf = nullptr;         // this rank's exchange buffer (peers write into it)
    uint64_t* words = nullptr;     // local device words (W_*)
    std::vector<void*> opened;     // IPC mappings of the peers' buffers
    uint64_t host_timeout_ns = 120000000000ull;
};

namespace {

int comm_error(ki_comm* c, int status, const char* fmt, const char* detail) {
    if (c && c->ctx) return ki::set_error(c->ctx, status, fmt, detail);
    return status;
}

// Bounded host-side wait for an NCCL call on a non-blocking communicator; aborts on timeout.
int nccl_wait(ki_comm* c, ncclResult_t r, const char* what) {
    const Nccl* N = nccl();
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
        if (r == ncclSuccess) return KI_OK;
        if (r != ncclInProgress) return comm_error(c, KI_ERR_NCCL, "%s", N->GetErrorString(r));
        const auto el = std::chrono::steady_clock::now() - t0;
        if ((uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(el).count() > c->host_timeout_ns) {
            N->CommAbort(c->nc);
            c->nc = nullptr;
            return comm_error(c, KI_ERR_TIMEOUT, "%s: NCCL did not complete in time (communicator aborted)", what);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
        if (N->CommGetAsyncError(c->nc, &r) != ncclSuccess) r = ncclSystemError;
    }
}

// Bounded host-side wait for a stream that runs NCCL work; aborts the communicator on timeout.
int stream_wait(ki_comm* c, cudaStream_t s, const char* what) {
    const Nccl* N = nccl();
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
        const cudaError_t q = cudaStreamQuery(s);
        if (q == cudaSuccess) return KI_OK;
        if (q != cudaErrorNotReady) return ki::cuda_error(c->ctx, q, what);
        ncclResult_t r = ncclSuccess;
        if (c->nc && N->CommGetAsyncError(c->nc, &r) == ncclSuccess && r != ncclSuccess && r != ncclInProgress)
            return comm_error(c, KI_ERR_NCCL, "%s", N->GetErrorString(r));
        const auto el = std::chrono::steady_clock::now() - t0;
        if ((uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(el).count() > c->host_timeout_ns) {
            if (c->nc) N->CommAbort(c->nc);
            c->nc = nullptr;
            return comm_error(c, KI_ERR_TIMEOUT, "%s: peers did not answer in time (communicator aborted)", what);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

// Device allocations shared by both kinds of communicator.
int comm_alloc(ki_comm* c) {
    KI_CUDA(c->ctx, cudaMalloc(&c->xbuf, kXBufBytes));
    KI_CUDA(c->ctx, cudaMemset(c->xbuf, 0, kXBufBytes));
    KI_CUDA(c->ctx, cudaMalloc(&c->words, W_WORDS * sizeof(uint64_t)));
    KI_CUDA(c->ctx, cudaMemset(c->words, 0, W_WORDS * sizeof(uint64_t)));
    KI_CUDA(c->ctx, cudaStreamCreateWithFlags(&c->setup, cudaStreamNonBlocking));
    return KI_OK;
}

// Keep the reason of a failed set-up for ki_last_error_string(NULL) before the context goes.
void keep_error(ki_comm* c, int rc) {
    char* t = ki::thread_error();
    if (c && c->ctx && c->ctx->last_error[0]) snprintf(t, 512, "%s", c->ctx->last_error);
    else snprintf(t, 512, "communicator set-up failed: %s", ki_status_string(rc));
    t[511] = 0;
}

void comm_free(ki_comm* c) {
    if (!c) return;
    if (c->ctx) {
        ki::DeviceGuard g(c->device);
        cudaDeviceSynchronize();
        for (void* p : c->opened) cudaIpcCloseMemHandle(p);
        if (c->xbuf) cudaFree(c->xbuf);
        if (c->words) cudaFree(c->words);
        if (c->setup) cudaStreamDestroy(c->setup);
    }
    if (c->nc) nccl()->CommDestroy(c->nc);
    if (c->ctx) ki_ctx_destroy(c->ctx);
    delete c;
}

int upload_peers(ki_comm* c, const std::vector<XSlot*>& bufs) {
    std::vector<uint64_t> h(kMaxRanks, 0);
    for (size_t i = 0; i < bufs.size(); ++i) h[i] = reinterpret_cast<uint64_t>(bufs[i]);
    KI_CUDA(c->ctx, cudaMemcpy(c->words + W_PEERS, h.data(), kMaxRanks * sizeof(uint64_t), cudaMemcpyHostToDevice));
    return KI_OK;
}

// Gather one RankRecord from every rank (multi-process set-up).
int gather_records(ki_comm* c, const RankRecord& mine, std::vector<RankRecord>& all) {
    const Nccl* N = nccl();
    RankRecord* d = nullptr;
    KI_CUDA(c->ctx, cudaMalloc(&d, sizeof(RankRecord) * (c->nranks + 1)));
    int rc = KI_OK;
    if (cudaMemcpy(d, &mine, sizeof(mine), cudaMemcpyHostToDevice) != cudaSuccess) rc = KI_ERR_CUDA;
    if (!rc) rc = nccl_wait(c, N->AllGather(d, d + 1, sizeof(RankRecord), ncclUint8, c->nc, c->setup), "ncclAllGather");
    if (!rc) rc = stream_wait(c, c->setup, "set-up all-gather");
    all.resize(c->nranks);
    if (!rc && cudaMemcpy(all.data(), d + 1, sizeof(RankRecord) * c->nranks, cudaMemcpyDeviceToHost) != cudaSuccess)
        rc = KI_ERR_CUDA;
    cudaFree(d);
    if (rc == KI_ERR_CUDA) return ki::set_error(c->ctx, KI_ERR_CUDA, "set-up all-gather: CUDA copy failed");
    return rc;
}

int exchange(ki_comm* c, int fold, const uint64_t* d_local, double* out_f64, float* out_f32, uint64_t* out_prefix,
             uint64_t* out_total, cudaStream_t s) {
    XArgs a;
    a.peers = nullptr;
    a.mine = c->xbuf;
    a.gathered = c->words + W_GATHERED;
    a.local = d_local;
    a.epoch = c->words + W_EPOCH;
    a.nranks = c->nranks;
    a.rank = c->rank;
    a.fold = fold;
    a.out_f64 = out_f64;
    a.out_f32 = out_f32;
    a.out_prefix = out_prefix;
    a.out_total = out_total;
    a.status = c->ctx->d_status;
    a.timeout_ns = c->ctx->wait_timeout_ns;
    if (c->exchange == KI_XCHG_PEER) {
        a.peers = reinterpret_cast<XSlot* const*>(c->words + W_PEERS);
    } else {
        const Nccl* N = nccl();
        int rc = nccl_wait(c, N->AllGather(d_local, c->words + W_GATHERED, 1, ncclUint64, c->nc, s), "ncclAllGather");
        if (rc) return rc;
    }
    exchange_kernel<<<1, 32, 0, s>>>(a);
    return ki::check_launch(c->ctx, "exchange_kernel launch");
}

#define KI_CHECK_COMM(c)                                                  \
    do {                                                                  \
        if (!(c) || !(c)->ctx) return KI_ERR_ARG;                         \
        if ((c)->exchange == KI_XCHG_NCCL && !(c)->nc)                    \
            return ki::set_error((c)->ctx, KI_ERR_NCCL, "communicator was aborted"); \
    } while (0)

}  // namespace

extern "C" {

int ki_comm_shard_range(size_t n, int nranks, int rank, size_t* lo, size_t* count) {
    if (nranks <= 0 || rank < 0 || rank >= nranks || !lo || !count) return KI_ERR_ARG;
    const size_t q = n / (size_t)nranks, r = n % (size_t)nranks;
    *lo = (size_t)rank * q + ((size_t)rank < r ? (size_t)rank : r);
    *count = q + ((size_t)rank < r ? 1 : 0);
    return KI_OK;
}

int ki_comm_scan_shard_range(size_t n, int nranks, int rank, size_t* lo, size_t* count) {
    if (nranks <= 0 || rank < 0 || rank >= nranks || !lo || !count) return KI_ERR_ARG;
    // weights 2, ..., 2, 3 (the last rank moves 16 B per element, the others 24): boundaries at
    // n * 2r / (2 nranks + 1), rounded down to 256 elements so every shard starts 2 KiB aligned
    auto edge = [&](int r) -> size_t {
        if (r >= nranks) return n;
        const unsigned __int128 e = (unsigned __int128)n * (unsigned)(2 * r) / (unsigned)(2 * nranks + 1);
        return (size_t)e & ~(size_t)255;
    };
    *lo = edge(rank);
    *count = edge(rank + 1) - *lo;
    return KI_OK;
}

int ki_comm_get_id(ki_comm_id* id) {
    if (!id) return KI_ERR_ARG;
    static_assert(sizeof(ncclUniqueId) <= sizeof(ki_comm_id), "ki_comm_id holds an ncclUniqueId");
    const Nccl* N = nccl();
    if (!N) return KI_ERR_UNSUPPORTED;
    ncclUniqueId u;
    if (N->GetUniqueId(&u) != ncclSuccess) return KI_ERR_NCCL;
    memset(id, 0, sizeof(*id));
    memcpy(id->internal, &u, sizeof(u));
    return KI_OK;
}

int ki_comm_init_rank(int device, int nranks, int rank, const ki_comm_id* id, int exchange, ki_comm** out) {
    if (!out) return KI_ERR_ARG;
    *out = nullptr;
    if (!id || nranks < 1 || nranks > kMaxRanks || rank < 0 || rank >= nranks) return KI_ERR_ARG;
    if (exchange != KI_XCHG_AUTO && exchange != KI_XCHG_PEER && exchange != KI_XCHG_NCCL) return KI_ERR_ARG;
    const Nccl* N = nccl();
    if (!N) return KI_ERR_UNSUPPORTED;
    ki_comm* c = new (std::nothrow) ki_comm();
    if (!c) return KI_ERR_NOMEM;
    c->nranks = nranks;
    c->rank = rank;
    c->device = device;
    c->multi_process = true;
    int rc = ki_ctx_create(device, &c->ctx);
    if (rc) {
        keep_error(nullptr, rc);
        delete c;
        return rc;
    }
    ki::DeviceGuard g(device);
    rc = comm_alloc(c);
    if (!rc) {
        ncclUniqueId u;
        memcpy(&u, id->internal, sizeof(u));
        ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
        cfg.blocking = 0;  // set-up waits are bounded on the host (nccl_wait)
        rc = nccl_wait(c, N->CommInitRankConfig(&c->nc, nranks, u, rank, &cfg), "ncclCommInitRankConfig");
    }
    // step 1: exchange buffers and GPU identities
    RankRecord mine;
    memset(&mine, 0, sizeof(mine));
    std::vector<RankRecord> all;
    if (!rc) {
        cudaDeviceProp p;
        if (cudaGetDeviceProperties(&p, device) != cudaSuccess) rc = KI_ERR_CUDA;
        else memcpy(mine.uuid, &p.uuid, 16);
    }
    if (!rc && exchange != KI_XCHG_NCCL && cudaIpcGetMemHandle(&mine.xbuf, c->xbuf) != cudaSuccess) {
        cudaGetLastError();
        if (exchange == KI_XCHG_PEER) rc = ki::set_error(c->ctx, KI_ERR_UNSUPPORTED, "cudaIpcGetMemHandle failed");
    }
    if (!rc) rc = gather_records(c, mine, all);
    if (!rc) {
        for (int i = 0; i < nranks && !rc; ++i)
            for (int j = i + 1; j < nranks && !rc; ++j)
                if (memcmp(all[i].uuid, all[j].uuid, 16) == 0)
                    rc = ki::set_error(c->ctx, KI_ERR_UNSUPPORTED,
                                       "ranks %d and %d share one GPU: their exchange waits would wait on one another",
                                       i, j);
    }
    // step 2: map every peer's buffer; all ranks agree on peer or NCCL exchange
    std::vector<XSlot*> bufs(nranks, nullptr);
    if (!rc) {
        int ok = exchange != KI_XCHG_NCCL;
        for (int q = 0; q < nranks && ok; ++q) {
            if (q == rank) {
                bufs[q] = c->xbuf;
                continue;
            }
            void* p = nullptr;
            if (cudaIpcOpenMemHandle(&p, all[q].xbuf, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
                cudaGetLastError();
                ok = 0;
            } else {
                c->opened.push_back(p);
                bufs[q] = static_cast<XSlot*>(p);
            }
        }
        RankRecord r2 = mine;
        r2.ipc_ok = ok;
        rc = gather_records(c, r2, all);
        bool every = true;
        for (int q = 0; q < nranks && !rc; ++q) every = every && all[q].ipc_ok;
        if (!rc) {
            if (every) {
                c->exchange = KI_XCHG_PEER;
                rc = upload_peers(c, bufs);
            } else if (exchange == KI_XCHG_PEER) {
                rc = ki::set_error(c->ctx, KI_ERR_UNSUPPORTED, "peer exchange requested but a peer buffer could not be mapped");
            } else {
                c->exchange = KI_XCHG_NCCL;
            }
        }
    }
    if (rc) {
        keep_error(c, rc);
        if (c->nc) {
            N->CommAbort(c->nc);
            c->nc = nullptr;
        }
        comm_free(c);
        return rc;
    }
    *out = c;
    return KI_OK;
}

int ki_comm_create(int ndev, const int* devs, ki_comm** comms) {
    if (!comms || !devs || ndev < 1 || ndev > kMaxRanks) return KI_ERR_ARG;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess) return KI_ERR_CUDA;
    for (int i = 0; i < ndev; ++i) {
        comms[i] = nullptr;
        if (devs[i] < 0 || devs[i] >= count) return KI_ERR_ARG;
        for (int j = 0; j < i; ++j)
            if (devs[i] == devs[j]) return KI_ERR_ARG;  // two ranks on one GPU would wait on one another
    }
    for (int i = 0; i < ndev; ++i)
        for (int j = 0; j < ndev; ++j) {
            int ok = 0;
            if (i != j && (cudaDeviceCanAccessPeer(&ok, devs[i], devs[j]) != cudaSuccess || !ok))
                return KI_ERR_UNSUPPORTED;
        }
    std::vector<ki_comm*> cs(ndev, nullptr);
    int rc = KI_OK;
    for (int i = 0; i < ndev && !rc; ++i) {
        ki_comm* c = new (std::nothrow) ki_comm();
        if (!c) {
            rc = KI_ERR_NOMEM;
            break;
        }
        cs[i] = c;
        c->nranks = ndev;
        c->rank = i;
        c->device = devs[i];
        c->exchange = KI_XCHG_PEER;
        rc = ki_ctx_create(devs[i], &c->ctx);
        if (rc) break;
        ki::DeviceGuard g(devs[i]);
        for (int j = 0; j < ndev; ++j) {
            if (j == i) continue;
            const cudaError_t e = cudaDeviceEnablePeerAccess(devs[j], 0);
            if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled) {
                rc = ki::cuda_error(c->ctx, e, "cudaDeviceEnablePeerAccess");
                break;
            }
            cudaGetLastError();  // clears cudaErrorPeerAccessAlreadyEnabled
        }
        if (!rc) rc = comm_alloc(c);
    }
    if (!rc) {
        std::vector<XSlot*> bufs(ndev);
        for (int i = 0; i < ndev; ++i) bufs[i] = cs[i]->xbuf;
        for (int i = 0; i < ndev && !rc; ++i) {
            ki::DeviceGuard g(devs[i]);
            rc = upload_peers(cs[i], bufs);
        }
    }
    if (rc) {
        for (ki_comm* c : cs)
            if (c && c->ctx && c->ctx->last_error[0]) keep_error(c, rc);
        for (ki_comm* c : cs) comm_free(c);
        return rc;
    }
    for (int i = 0; i < ndev; ++i) comms[i] = cs[i];
    return KI_OK;
}

int ki_comm_destroy(ki_comm* comm) {
    if (!comm) return KI_OK;
    int rc = KI_OK;
    if (comm->multi_process && comm->nc) {
        // every rank must be done with the others' buffers before any is unmapped or freed
        ki::DeviceGuard g(comm->device);
        cudaDeviceSynchronize();
        RankRecord r;
        memset(&r, 0, sizeof(r));
        std::vector<RankRecord> all;
        rc = gather_records(comm, r, all);
        if (!rc) rc = nccl_wait(comm, nccl()->CommFinalize(comm->nc), "ncclCommFinalize");
        if (rc && comm->nc) {
            nccl()->CommAbort(comm->nc);
            comm->nc = nullptr;
        }
    }
    comm_free(comm);
    return rc;
}

int ki_comm_abort(ki_comm* comm) {
    if (!comm) return KI_OK;
    if (comm->nc) {
        nccl()->CommAbort(comm->nc);
        comm->nc = nullptr;
    }
    comm_free(comm);
    return KI_OK;
}

int ki_comm_info(const ki_comm* comm, int* nranks, int* rank, int* device, int* exchange) {
    if (!comm) return KI_ERR_ARG;
    if (nranks) *nranks = comm->nranks;
    if (rank) *rank = comm->rank;
    if (device) *device = comm->device;
    if (exchange) *exchange = comm->exchange;
    return KI_OK;
}

int ki_comm_get_ctx(ki_comm* comm, ki_ctx** ctx) {
    if (!comm || !ctx) return KI_ERR_ARG;
    *ctx = comm->ctx;
    return KI_OK;
}

int ki_reduce_sum_f32_sharded(ki_comm* comm, const float* d_x, size_t n_local, float* d_out_f32, double* d_out_f64,
                              void* stream) {
    KI_CHECK_COMM(comm);
    if (!d_out_f32 && !d_out_f64) return ki::set_error(comm->ctx, KI_ERR_ARG, "reduce: no output");
    if (comm->nranks == 1) return ki_reduce_sum_f32(comm->ctx, d_x, n_local, d_out_f32, d_out_f64, stream);
    KI_GUARD(comm->ctx);
    cudaStream_t s = ki::as_stream(stream);
    double* part = reinterpret_cast<double*>(comm->words + W_LOCAL);
    int rc = ki_reduce_sum_f32(comm->ctx, d_x, n_local, nullptr, part, stream);
    if (rc) return rc;
    return exchange(comm, XF_SUM_F64, comm->words + W_LOCAL, d_out_f64, d_out_f32, nullptr, nullptr, s);
}

int ki_scan_inclusive_i64_sharded(ki_comm* comm, const int64_t* d_in, int64_t* d_out, size_t n_local, void* stream) {
    KI_CHECK_COMM(comm);
    if (comm->nranks == 1) return ki_scan_inclusive_i64(comm->ctx, d_in, d_out, n_local, 0, stream);
    KI_GUARD(comm->ctx);
    cudaStream_t s = ki::as_stream(stream);
    int64_t* total = reinterpret_cast<int64_t*>(comm->words + W_LOCAL);
    int64_t* seed = reinterpret_cast<int64_t*>(comm->words + W_SEED);
    // nothing after the exchange may block: phase 2's scratch and kernel are made ready first
    int rc = ki_scan_i64_reserve(comm->ctx, n_local);
    if (rc) return rc;
    if (comm->rank == comm->nranks - 1) {  // nobody reads the last shard's total: publish 0 unread
        KI_CUDA(comm->ctx, cudaMemsetAsync(total, 0, sizeof(int64_t), s));
    } else {
        rc = ki_reduce_sum_i64(comm->ctx, d_in, n_local, total, stream);
    }
    if (rc) return rc;
    rc = exchange(comm, XF_PREFIX_I64, comm->words + W_LOCAL, nullptr, nullptr, comm->words + W_SEED, nullptr, s);
    if (rc) return rc;
    return ki_scan_inclusive_i64_dseed(comm->ctx, d_in, d_out, n_local, seed, stream);
}

int ki_scan_inclusive_i64_sharded_host(ki_comm* comm, const int64_t* h_in, int64_t* h_out, size_t n_local,
                                       void* stream) {
    KI_CHECK_COMM(comm);
    ki_ctx* ctx = comm->ctx;
    if (n_local > 0 && (!h_in || !h_out)) return ki::set_error(ctx, KI_ERR_ARG, "scan_host: null pointer");
    if (!ki::aligned(h_in, 8) || !ki::aligned(h_out, 8))
        return ki::set_error(ctx, KI_ERR_ARG, "scan_host: Int64 pointers must be 8-byte aligned");
    if (comm->nranks == 1) return ki_scan_inclusive_i64_host(ctx, h_in, h_out, n_local, 0, stream);
    KI_GUARD(ctx);
    int rc = ki_ensure_pipe(ctx);
    if (rc) return rc;
    constexpr size_t kChunk = KI_PIPE_CHUNK / sizeof(int64_t);
    const size_t nch = (n_local + kChunk - 1) / kChunk;
    void* shard = nullptr;
    void* parts = nullptr;
    rc = ki::ensure_region(ctx, KI_REG_HOST_SHARD, n_local * sizeof(int64_t), &shard);
    if (!rc) rc = ki::ensure_region(ctx, KI_REG_HOST_PART, (nch + 1) * sizeof(int64_t), &parts);
    if (!rc) rc = ki_scan_i64_reserve(ctx, kChunk);  // phase 2 (after the exchange) must not block
    if (rc) return rc;
    int64_t* buf = static_cast<int64_t*>(shard);
    int64_t* part = static_cast<int64_t*>(parts);
    cudaStream_t s = ki::as_stream(stream);
    cudaStream_t up = ctx->pipe_stream[0], kern = ctx->pipe_stream[1], down = ctx->pipe_stream[2];
    KI_CUDA(ctx, cudaEventRecord(ctx->pipe_begin, s));
    for (int i = 0; i < 3; ++i) KI_CUDA(ctx, cudaStreamWaitEvent(ctx->pipe_stream[i], ctx->pipe_begin, 0));
    // phase 1: the shard comes in chunk by chunk, each chunk summed as soon as it has landed
    for (size_t i = 0; i < nch; ++i) {
        const int k = (int)(i % KI_PIPE_SLOTS);
        const size_t off = i * kChunk, len = (n_local - off < kChunk) ? n_local - off : kChunk;
        KI_CUDA(ctx, cudaMemcpyAsync(buf + off, h_in + off, len * sizeof(int64_t), cudaMemcpyHostToDevice, up));
        KI_CUDA(ctx, cudaEventRecord(ctx->pipe_landed[k], up));
        KI_CUDA(ctx, cudaStreamWaitEvent(kern, ctx->pipe_landed[k], 0));
        rc = ki_reduce_sum_i64(ctx, buf + off, len, part + i, kern);
        if (rc) return rc;
    }
    int64_t* total = reinterpret_cast<int64_t*>(comm->words + W_LOCAL);
    rc = ki_reduce_sum_i64(ctx, part, nch, total, kern);  // chunk totals in order (wrapping: exact)
    if (!rc) rc = exchange(comm, XF_PREFIX_I64, comm->words + W_LOCAL, nullptr, nullptr, comm->words + W_SEED, nullptr,
                           kern);
    if (rc) return rc;
    // phase 2: scan in place chunk by chunk (chunk i seeded with chunk i-1's last output) and send back
    for (size_t i = 0; i < nch; ++i) {
        const int k = (int)(i % KI_PIPE_SLOTS);
        const size_t off = i * kChunk, len = (n_local - off < kChunk) ? n_local - off : kChunk;
        const int64_t* seed = i == 0 ? reinterpret_cast<const int64_t*>(comm->words + W_SEED) : buf + off - 1;
        rc = ki_scan_inclusive_i64_dseed(ctx, buf + off, buf + off, len, seed, kern);
        if (rc) return rc;
        KI_CUDA(ctx, cudaEventRecord(ctx->pipe_copied[k], kern));
        KI_CUDA(ctx, cudaStreamWaitEvent(down, ctx->pipe_copied[k], 0));
        KI_CUDA(ctx, cudaMemcpyAsync(h_out + off, buf + off, len * sizeof(int64_t), cudaMemcpyDeviceToHost, down));
    }
    KI_CUDA(ctx, cudaEventRecord(ctx->pipe_end, kern));
    KI_CUDA(ctx, cudaStreamWaitEvent(down, ctx->pipe_end, 0));
    KI_CUDA(ctx, cudaEventRecord(ctx->pipe_end, down));
    KI_CUDA(ctx, cudaStreamWaitEvent(s, ctx->pipe_end, 0));
    return KI_OK;
}

int ki_compact_gt_f32_sharded(ki_comm* comm, const float* d_x, size_t n_local, float threshold, float* d_out_vals,
                              int32_t* d_out_idx, int64_t index_base, uint64_t* d_count, uint64_t* d_offset,
                              uint64_t* d_total, void* stream) {
    KI_CHECK_COMM(comm);
    if (n_local > 0 && !d_out_vals && !d_out_idx) return ki::set_error(comm->ctx, KI_ERR_ARG, "compact: no output");
    KI_GUARD(comm->ctx);
    cudaStream_t s = ki::as_stream(stream);
    uint64_t* cnt = d_count ? d_count : comm->words + W_COUNT;
    if (n_local == 0) {  // an empty shard keeps nothing but still takes part in the exchange
        KI_CUDA(comm->ctx, cudaMemsetAsync(cnt, 0, sizeof(uint64_t), s));
    } else {
        int rc = ki_compact_gt_f32(comm->ctx, d_x, n_local, threshold, d_out_vals, d_out_idx, index_base, cnt, stream);
        if (rc) return rc;
    }
    return exchange(comm, XF_PREFIX_U64, cnt, nullptr, nullptr, d_offset ? d_offset : comm->words + W_OFFSET,
                    d_total ? d_total : comm->words + W_TOTAL, s);
}

}  // extern "C"
