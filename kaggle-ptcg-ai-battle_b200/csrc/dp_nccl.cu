// Native data-parallel exchange of the PPO step: the gradient average fused
// with a sharded Adam, issued by the library itself over NCCL.
//
// The reference trainer all-reduces the whole grad arena once after backward
// and every rank runs the optimizer over all of it (native/src/muon.cu:
// 209-214).  Here each final gradient span that backward produces (the same
// layer-ordered spans the grad hook reports, in backward order) is
// reduce-scattered on a communication stream while the rest of backward runs;
// after backward each rank clips with the global norm (one fp64 all-reduce),
// runs Adam on its own pieces only, and the updated master weights are
// all-gathered span by span.  Reduce-scatter + all-gather move what one
// all-reduce moves, and the optimizer reads and writes 1/world of the arena.
//
// NCCL is opened at run time (dlopen of libnccl.so.2, or $PTCG_NCCL_LIB), so
// the library loads and runs single-GPU work on hosts without NCCL; in a
// process that already loaded NCCL (torch does) the same instance is reused.
// Only the communicator's own collectives are issued: no peer-memory loads,
// no TMA multicast.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <algorithm>
#include <cstring>
#include <mutex>
#include <vector>

#include "internal.h"

namespace {

struct NcclApi {
    void* h = nullptr;
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*ReduceScatter)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t,
                                  ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t,
                              ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

NcclApi g_nccl;
std::mutex g_nccl_mu;
thread_local char g_dp_err[512];

void dp_set_err(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_dp_err, sizeof g_dp_err, fmt, ap);
    va_end(ap);
}

template <class F>
bool sym(void* h, const char* name, F& f) {
    f = (F)dlsym(h, name);
    return f != nullptr;
}

bool nccl_load() {
    std::lock_guard<std::mutex> lk(g_nccl_mu);
    if (g_nccl.h) return true;
    const char* env = getenv("PTCG_NCCL_LIB");
    const char* name = env && *env ? env : "libnccl.so.2";
    void* h = dlopen(name, RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
        dp_set_err("cannot open NCCL (%s): %s", name, dlerror());
        return false;
    }
    NcclApi a;
    a.h = h;
    bool ok = sym(h, "ncclGetUniqueId", a.GetUniqueId) && sym(h, "ncclCommInitRank", a.CommInitRank) &&
              sym(h, "ncclCommDestroy", a.CommDestroy) && sym(h, "ncclCommAbort", a.CommAbort) &&
              sym(h, "ncclReduceScatter", a.ReduceScatter) && sym(h, "ncclAllGather", a.AllGather) &&
              sym(h, "ncclAllReduce", a.AllReduce) && sym(h, "ncclGroupStart", a.GroupStart) &&
              sym(h, "ncclGroupEnd", a.GroupEnd) && sym(h, "ncclGetErrorString", a.GetErrorString);
    if (!ok) {
        dp_set_err("NCCL library %s lacks a required symbol", name);
        dlclose(h);
        return false;
    }
    g_nccl = a;
    return true;
}

#define NC(x) do { ncclResult_t _r = (x); if (_r != ncclSuccess) { \
    dp_set_err("%s failed: %s", #x, g_nccl.GetErrorString(_r)); return 1; } } while (0)
#define CU(x) do { cudaError_t _e = (x); if (_e != cudaSuccess) { \
    dp_set_err("%s failed: %s", #x, cudaGetErrorString(_e)); return 1; } } while (0)

// [v, ~v] of a 64-bit checksum held as two uint32 halves, as int64
__global__ void k_ck_pack(long long* both, const unsigned int* ck) {
    const long long v = (long long)(((unsigned long long)ck[1] << 32) | ck[0]);
    both[0] = v;
    both[1] = ~v;
}

__global__ void k_ck_unpack(long long* minmax, const long long* both) {
    minmax[0] = ~both[1];
    minmax[1] = both[0];
}

}  // namespace

// One span of the grad arena: this rank's piece of it is [rank * c,
// rank * c + c) clipped to count, held in the shard at soff.
struct DpBucket {
    long off = 0, count = 0, c = 0, soff = 0;
    float* send = nullptr;      // world * c floats, zero past count
    float* gather = nullptr;    // world * c floats
    float* piece = nullptr;     // c floats
};

struct DpState {
    int rank = 0, world = 1, dev = 0;
    ncclComm_t comm = nullptr;
    cudaStream_t cs = nullptr;
    cudaEvent_t ev = nullptr, ev_join = nullptr;
    std::vector<DpBucket> b;
    void* base = nullptr;       // one allocation for every buffer below
    float* shard = nullptr;
    long used = 0;
    long* seg = nullptr;        // {arena offset, shard offset, length} per piece
    int nseg = 0;
    double* sumsq = nullptr;
    long long* ck = nullptr;    // [v, ~v]
    int pending = 0;            // spans reduce-scattered since the last join
};

const char* dp_last_error() { return g_dp_err; }

int dp_unique_id(void* out128) {
    if (!nccl_load()) return 1;
    static_assert(sizeof(ncclUniqueId) == DP_UID_BYTES, "ncclUniqueId size");
    ncclUniqueId id;
    NC(g_nccl.GetUniqueId(&id));
    memcpy(out128, &id, sizeof id);
    return 0;
}

static int dp_alloc(DpState* d) {
    // layout: per bucket send + gather + piece, then shard, seg, sumsq, ck
    size_t floats = 0;
    for (auto& k : d->b) floats += (size_t)(2 * d->world + 1) * k.c;
    floats += (size_t)d->used;
    size_t bytes = ((floats * 4 + 255) / 256) * 256;
    size_t seg_off = bytes;
    bytes += ((size_t)d->b.size() * 3 * 8 + 255) / 256 * 256;
    size_t ss_off = bytes;
    bytes += 256;
    CU(cudaMalloc(&d->base, bytes));
    CU(cudaMemset(d->base, 0, bytes));
    float* f = (float*)d->base;
    for (auto& k : d->b) {
        k.send = f; f += (size_t)d->world * k.c;
        k.gather = f; f += (size_t)d->world * k.c;
        k.piece = f; f += k.c;
    }
    d->shard = f;
    d->seg = (long*)((char*)d->base + seg_off);
    d->sumsq = (double*)((char*)d->base + ss_off);
    d->ck = (long long*)((char*)d->base + ss_off + 64);
    std::vector<long> seg;
    for (auto& k : d->b) {
        long start = (long)d->rank * k.c;
        long len = std::min(k.count - start, k.c);
        if (len > 0) {
            seg.push_back(k.off + start);
            seg.push_back(k.soff);
            seg.push_back(len);
        }
    }
    d->nseg = (int)(seg.size() / 3);
    if (!seg.empty())
        CU(cudaMemcpy(d->seg, seg.data(), seg.size() * 8, cudaMemcpyHostToDevice));
    return 0;
}

int dp_create(DpState** out, const void* uid, int rank, int world, int dev, const long* spans,
              int nspans, long n_arena) {
    *out = nullptr;
    if (world < 1 || rank < 0 || rank >= world) {
        dp_set_err("bad rank %d / world %d", rank, world);
        return 1;
    }
    // the spans must tile [0, n_arena) exactly once
    {
        std::vector<std::pair<long, long>> v;
        for (int i = 0; i < nspans; i++) v.push_back({spans[2 * i], spans[2 * i + 1]});
        std::sort(v.begin(), v.end());
        long cur = 0;
        for (auto& p : v) {
            if (p.first != cur || p.second <= 0) {
                dp_set_err("gradient spans do not tile the arena (gap or overlap at %ld)", cur);
                return 1;
            }
            cur += p.second;
        }
        if (cur != n_arena) {
            dp_set_err("gradient spans cover %ld of %ld arena floats", cur, n_arena);
            return 1;
        }
    }
    if (!nccl_load()) return 1;
    DpState* d = new DpState();
    d->rank = rank; d->world = world; d->dev = dev;
    for (int i = 0; i < nspans; i++) {
        DpBucket k;
        k.off = spans[2 * i];
        k.count = spans[2 * i + 1];
        k.c = ((k.count + world - 1) / world + 3) / 4 * 4;     // 16-byte pieces
        k.soff = d->used;
        d->used += k.c;
        d->b.push_back(k);
    }
    int rc = 0;
    if (cudaSetDevice(dev) != cudaSuccess || dp_alloc(d)) rc = 1;
    if (!rc && (cudaStreamCreateWithFlags(&d->cs, cudaStreamNonBlocking) != cudaSuccess ||
                cudaEventCreateWithFlags(&d->ev, cudaEventDisableTiming) != cudaSuccess ||
                cudaEventCreateWithFlags(&d->ev_join, cudaEventDisableTiming) != cudaSuccess)) {
        dp_set_err("stream / event creation failed");
        rc = 1;
    }
    if (!rc) {
        ncclUniqueId id;
        memcpy(&id, uid, sizeof id);
        ncclResult_t r = g_nccl.CommInitRank(&d->comm, world, id, rank);
        if (r != ncclSuccess) {
            dp_set_err("ncclCommInitRank (rank %d of %d) failed: %s", rank, world,
                       g_nccl.GetErrorString(r));
            d->comm = nullptr;
            rc = 1;
        }
    }
    if (rc) {
        char keep[sizeof g_dp_err];
        memcpy(keep, g_dp_err, sizeof keep);
        dp_destroy(d, true);
        memcpy(g_dp_err, keep, sizeof keep);
        return 1;
    }
    *out = d;
    return 0;
}

void dp_destroy(DpState* d, bool abort) {
    if (!d) return;
    cudaSetDevice(d->dev);
    if (d->comm) {
        if (abort) g_nccl.CommAbort(d->comm);
        else {
            if (d->cs) cudaStreamSynchronize(d->cs);
            g_nccl.CommDestroy(d->comm);
        }
    }
    if (d->cs) cudaStreamSynchronize(d->cs);
    if (d->ev) cudaEventDestroy(d->ev);
    if (d->ev_join) cudaEventDestroy(d->ev_join);
    if (d->cs) cudaStreamDestroy(d->cs);
    if (d->base) cudaFree(d->base);
    delete d;
}

// Start the reduce-scatter of one final span, ordered after the work issued
// so far on the compute stream s.
int dp_bucket(DpState* d, const float* grads, long off, long count, cudaStream_t s) {
    DpBucket* k = nullptr;
    for (auto& q : d->b)
        if (q.off == off) { k = &q; break; }
    if (!k || k->count != count) {
        dp_set_err("gradient span [%ld, +%ld) is not one planned at dp init", off, count);
        return 1;
    }
    CU(cudaEventRecord(d->ev, s));
    CU(cudaStreamWaitEvent(d->cs, d->ev, 0));
    CU(cudaMemcpyAsync(k->send, grads + off, (size_t)count * 4, cudaMemcpyDeviceToDevice, d->cs));
    NC(g_nccl.ReduceScatter(k->send, d->shard + k->soff, (size_t)k->c, ncclFloat32, ncclAvg,
                            d->comm, d->cs));
    d->pending++;
    return 0;
}

int dp_join(DpState* d, cudaStream_t s, int* spans_seen) {
    if (spans_seen) *spans_seen = d->pending;
    d->pending = 0;
    CU(cudaEventRecord(d->ev_join, d->cs));
    CU(cudaStreamWaitEvent(s, d->ev_join, 0));
    return 0;
}

int dp_nbuckets(DpState* d) { return (int)d->b.size(); }

float* dp_shard(DpState* d, long* used, const long** seg, int* nseg, double** sumsq) {
    *used = d->used;
    *seg = d->seg;
    *nseg = d->nseg;
    *sumsq = d->sumsq;
    return d->shard;
}

int dp_allreduce_sum_f64(DpState* d, double* x, cudaStream_t s) {
    NC(g_nccl.AllReduce(x, x, 1, ncclFloat64, ncclSum, d->comm, s));
    return 0;
}

// The updated master weights: each rank's pieces out of params, all-gathered
// (one NCCL group), then every span written back whole.
int dp_gather_params(DpState* d, float* params, cudaStream_t s) {
    for (auto& k : d->b) {
        long start = (long)d->rank * k.c;
        long len = std::min(k.count - start, k.c);
        if (len > 0)
            CU(cudaMemcpyAsync(k.piece, params + k.off + start, (size_t)len * 4,
                               cudaMemcpyDeviceToDevice, s));
    }
    NC(g_nccl.GroupStart());
    for (auto& k : d->b) {
        ncclResult_t r = g_nccl.AllGather(k.piece, k.gather, (size_t)k.c, ncclFloat32, d->comm, s);
        if (r != ncclSuccess) {
            g_nccl.GroupEnd();
            dp_set_err("ncclAllGather failed: %s", g_nccl.GetErrorString(r));
            return 1;
        }
    }
    NC(g_nccl.GroupEnd());
    for (auto& k : d->b)
        CU(cudaMemcpyAsync(params + k.off, k.gather, (size_t)k.count * 4, cudaMemcpyDeviceToDevice,
                           s));
    return 0;
}

// min / max over ranks of a 64-bit checksum in one collective: MAX of
// [v, ~v] (bitwise not reverses the order of two's-complement integers, so
// min = ~max(~v)).  Written to minmax_dev[0..1] in stream order, no host wait.
int dp_weights_agree(DpState* d, const unsigned int* ck_dev, long long* minmax_dev,
                     cudaStream_t s) {
    ++g_ptcg_launches, k_ck_pack<<<1, 1, 0, s>>>(d->ck, ck_dev);
    CU(cudaGetLastError());
    NC(g_nccl.AllReduce(d->ck, d->ck, 2, ncclInt64, ncclMax, d->comm, s));
    ++g_ptcg_launches, k_ck_unpack<<<1, 1, 0, s>>>(minmax_dev, d->ck);
    CU(cudaGetLastError());
    return 0;
}
