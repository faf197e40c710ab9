// dp.cu — data parallelism for the training step: one process per GPU, the
// gradient arena all-reduced (sum) over NCCL in buckets that are launched on a
// high-priority communication stream as soon as the backward has finished
// their layers, so the exchange overlaps the rest of the backward.  The
// reference is single-GPU (src/main.cpp:54); this has no counterpart there.
//
// Communicators are created non-blocking (ncclCommInitRankConfig with
// blocking = 0) and watched: a host thread checks every enqueued collective
// against a deadline and polls ncclCommGetAsyncError; on a timeout (a peer that
// left, a hung link) or an asynchronous NCCL error it aborts the communicators
// (ncclCommAbort ends NCCL kernels still waiting on a peer), and every later
// call on the model returns RBK_ERR_TIMEOUT / RBK_ERR_NCCL instead of hanging.
//
// Two communicators share the ranks: the buckets that overlap the backward use
// one whose CTA count is capped (NCCL's CTAs otherwise take SMs from the
// persistent tcgen05 GEMM grids), the last bucket — the embeddings, reduced
// after the backward has ended, with nothing left to overlap — uses one
// without the cap.
#include <algorithm>
#include <chrono>
#include <cstring>
#include <deque>
#include <mutex>
#include <thread>

#include "model.h"

namespace rbk {

using Clock = std::chrono::steady_clock;

struct DpWatch {
    std::thread th;
    std::mutex mu;
    bool stop = false;
    int device = 0;
    double timeout_s = 300.0;
    int failed = RBK_OK;                       // guarded by mu
    ncclComm_t comms[2] = {nullptr, nullptr};  // guarded by mu; nulled after an abort
    std::deque<std::pair<cudaEvent_t, Clock::time_point>> pending;
    std::vector<cudaEvent_t> spare;
    std::vector<cudaEvent_t> all;

    // Under mu: abort both communicators (NCCL kernels waiting on a peer exit).
    void abort_locked(int why) {
        if (failed == RBK_OK) failed = why;
        if (comms[1] && comms[1] != comms[0]) ncclCommAbort(comms[1]);
        if (comms[0]) ncclCommAbort(comms[0]);
        comms[0] = comms[1] = nullptr;
    }

    void loop() {
        cudaSetDevice(device);
        while (true) {
            {
                std::lock_guard<std::mutex> lk(mu);
                if (stop) return;
                if (failed == RBK_OK) {
                    const auto now = Clock::now();
                    while (!pending.empty()) {
                        const cudaError_t q = cudaEventQuery(pending.front().first);
                        if (q == cudaSuccess) {
                            spare.push_back(pending.front().first);
                            pending.pop_front();
                            continue;
                        }
                        if (q != cudaErrorNotReady) {           // a sticky CUDA error: stop waiting on it
                            abort_locked(RBK_ERR_CUDA);
                            break;
                        }
                        const double waited = std::chrono::duration<double>(now - pending.front().second).count();
                        if (waited > timeout_s) abort_locked(RBK_ERR_TIMEOUT);
                        break;
                    }
                    for (int i = 0; i < 2 && failed == RBK_OK; ++i) {
                        if (!comms[i]) continue;
                        ncclResult_t ae = ncclSuccess;
                        if (ncclCommGetAsyncError(comms[i], &ae) != ncclSuccess ||
                            (ae != ncclSuccess && ae != ncclInProgress))
                            abort_locked(RBK_ERR_NCCL);
                    }
                }
            }
            std::this_thread::sleep_for(std::chrono::milliseconds(20));
        }
    }
};

namespace {

double env_double(const char* name, double dflt) {
    const char* e = getenv(name);
    return e && *e ? atof(e) : dflt;
}

// Host-side bound for a non-blocking communicator's own setup work: creation, the split, and
// the first collectives, which connect the ranks' channels (seconds on a large job).  The
// watchdog's deadline bounds collectives on the GPU, which may be much shorter.
constexpr double kSetupBoundS = 120.0;

// Wait (host) until a non-blocking communicator has finished its pending work.
ncclResult_t settle(ncclComm_t c, double timeout_s) {
    const auto t0 = Clock::now();
    ncclResult_t st = ncclInProgress;
    while (true) {
        if (ncclCommGetAsyncError(c, &st) != ncclSuccess) return ncclInternalError;
        if (st != ncclInProgress) return st;
        if (std::chrono::duration<double>(Clock::now() - t0).count() > timeout_s) return ncclInProgress;
        std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
}

// Units in backward order: 0 = ln_f + lm head (end of the arena), 1..L =
// layers L-1..0, L+1 = embeddings (start of the arena).  Each unit's range is
// contiguous.
void unit_range(const std::vector<rbk_tensor>& tab, int64_t n, const rbk_config* c, int u, int64_t* b, int64_t* e) {
    const int L = c->L;
    if (u == 0) { *b = tab[rbk_tail_tensor(c, 0)].offset; *e = n; return; }
    if (u == L + 1) { *b = 0; *e = tab[rbk_layer_tensor(0, 0)].offset; return; }
    const int l = L - u;
    *b = tab[rbk_layer_tensor(l, 0)].offset;
    *e = (l + 1 < L) ? tab[rbk_layer_tensor(l + 1, 0)].offset : tab[rbk_tail_tensor(c, 0)].offset;
}

// Enqueue one collective on stream st through communicator `tail ? uncapped : capped` and
// register it with the watchdog.  issue(comm) makes the NCCL call.
template <typename F>
int collective(DpState& d, bool tail, cudaStream_t st, const char* what, F issue) {
    DpWatch& w = *d.watch;
    std::lock_guard<std::mutex> lk(w.mu);
    if (w.failed != RBK_OK) {
        set_error("data parallel: the communicator was aborted (%s)",
                  w.failed == RBK_ERR_TIMEOUT ? "a collective timed out" : "an NCCL / CUDA error");
        return w.failed;
    }
    ncclComm_t c = w.comms[tail ? 1 : 0];
    ncclResult_t r = issue(c);
    if (r == ncclInProgress) r = settle(c, std::max(w.timeout_s, kSetupBoundS));
    if (r != ncclSuccess) {
        set_error("%s failed: %s", what, ncclGetErrorString(r));
        w.abort_locked(r == ncclInProgress ? RBK_ERR_TIMEOUT : RBK_ERR_NCCL);
        return w.failed;
    }
    cudaEvent_t ev;
    if (!w.spare.empty()) {
        ev = w.spare.back();
        w.spare.pop_back();
    } else {
        RBK_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
        w.all.push_back(ev);
    }
    RBK_CUDA(cudaEventRecord(ev, st));
    w.pending.emplace_back(ev, Clock::now());
    return RBK_OK;
}

int allreduce(DpState& d, float* buf, size_t n, bool tail) {
    return collective(d, tail, d.stream, "ncclAllReduce", [&](ncclComm_t c) {
        return ncclAllReduce(buf, buf, n, ncclFloat32, ncclSum, c, d.stream);
    });
}

// Sharded optimizer: reduce-scatter bucket [b, e) of the gradients in place (this rank's slice
// receives the sum over ranks), then clear the rest of the bucket, which still holds this
// rank's own unreduced gradients and must be zero for the next accumulation.
int reduce_scatter(rbk_model* m, int64_t b, int64_t e, bool tail) {
    DpState& d = m->dp;
    const size_t cnt = (size_t)((e - b) / d.world);
    float* base = m->grad + b;
    RBK_TRY(collective(d, tail, d.stream, "ncclReduceScatter", [&](ncclComm_t c) {
        return ncclReduceScatter(base, base + (size_t)d.rank * cnt, cnt, ncclFloat32, ncclSum, c, d.stream);
    }));
    if (d.rank > 0) RBK_CUDA(cudaMemsetAsync(base, 0, sizeof(float) * cnt * d.rank, d.stream));
    if (d.rank + 1 < d.world)
        RBK_CUDA(cudaMemsetAsync(base + cnt * (d.rank + 1), 0, sizeof(float) * cnt * (d.world - 1 - d.rank),
                                 d.stream));
    return RBK_OK;
}

// In-place all-gather of bucket [b, e) of an arena on stream st (each rank contributes its slice).
template <typename T>
int all_gather(rbk_model* m, T* arena, int64_t b, int64_t e, ncclDataType_t type, bool tail, cudaStream_t st) {
    DpState& d = m->dp;
    const size_t cnt = (size_t)((e - b) / d.world);
    T* base = arena + b;
    return collective(d, tail, st, "ncclAllGather", [&](ncclComm_t c) {
        return ncclAllGather(base + (size_t)d.rank * cnt, base, cnt, type, c, st);
    });
}

}  // namespace

// Bucket plan: walk the units in backward order, growing a pending range
// downwards through the arena, and close a bucket once it holds at least
// bucket_elems (the embeddings unit always closes the last one).  Pure host
// code: identical on every rank for the same configuration.
std::vector<DpBucket> dp_plan(const rbk_config* c, int64_t bucket_elems) {
    std::vector<rbk_tensor> tab(rbk_num_tensors(c));
    const int64_t n = rbk_param_table(c, tab.data());
    std::vector<DpBucket> out;
    int64_t pend_end = n;
    for (int u = 0; u <= c->L + 1; ++u) {
        int64_t b, e;
        unit_range(tab, n, c, u, &b, &e);
        if (pend_end - b >= bucket_elems || u == c->L + 1) {
            out.push_back(DpBucket{u, b, pend_end});
            pend_end = b;
        }
    }
    return out;
}

// Called by the backward after unit u's gradients are final on stream st.
int dp_unit_done(rbk_model* m, int u, cudaStream_t st) {
    DpState& d = m->dp;
    for (const DpBucket& bk : d.plan) {
        if (bk.unit != u) continue;
        RBK_CUDA(cudaEventRecord(d.layer_done[u], st));
        RBK_CUDA(cudaStreamWaitEvent(d.stream, d.layer_done[u], 0));
        if (d.shard)
            RBK_TRY(reduce_scatter(m, bk.begin, bk.end, u == m->cfg.L + 1));
        else
            RBK_TRY(allreduce(d, m->grad + bk.begin, (size_t)(bk.end - bk.begin), u == m->cfg.L + 1));
    }
    if (u == m->cfg.L + 1) {
        RBK_CUDA(cudaEventRecord(d.all_done, d.stream));
        RBK_CUDA(cudaStreamWaitEvent(st, d.all_done, 0));
    }
    return RBK_OK;
}

// One all-reduce of a whole gradient buffer, ordered after the work on st so far, with st
// waiting for it (the LoRA adapter arena).
int dp_reduce_all(rbk_model* m, float* buf, int64_t n, cudaStream_t st) {
    DpState& d = m->dp;
    RBK_CUDA(cudaEventRecord(d.layer_done[0], st));
    RBK_CUDA(cudaStreamWaitEvent(d.stream, d.layer_done[0], 0));
    RBK_TRY(allreduce(d, buf, (size_t)n, true));
    RBK_CUDA(cudaEventRecord(d.all_done, d.stream));
    RBK_CUDA(cudaStreamWaitEvent(st, d.all_done, 0));
    return RBK_OK;
}

// Sharded optimizer step on stream st: phase 1 of the tail over this rank's slices (overflow
// flag and per-tensor sums of squares into xbuf), one small all-reduce of xbuf so every rank
// takes the same skip decision and clip factors, phase 2 over the slices, then the FP16
// weights all-gathered bucket by bucket on the communication stream, in forward order
// (embeddings first), each bucket's completion recorded for dp_wait_weights.
int dp_optimizer_step(rbk_model* m, const rbk_tail_args* a, cudaStream_t st) {
    DpState& d = m->dp;
    const int nx = 1 + (a->max_norm > 0.0f ? a->nseg : 0);
    RBK_TRY(tail_launch(m->ctx, a, d.own, 1, d.xbuf, st));
    RBK_TRY(collective(d, true, st, "ncclAllReduce", [&](ncclComm_t c) {
        return ncclAllReduce(d.xbuf, d.xbuf, (size_t)nx, ncclFloat32, ncclSum, c, st);
    }));
    RBK_TRY(tail_launch(m->ctx, a, d.own, 2, d.xbuf, st));
    d.masters_partial = true;
    RBK_CUDA(cudaEventRecord(d.tail_done, st));
    RBK_CUDA(cudaStreamWaitEvent(d.stream, d.tail_done, 0));
    for (int i = (int)d.plan.size() - 1; i >= 0; --i) {
        const DpBucket& bk = d.plan[i];
        RBK_TRY(all_gather(m, m->p16, bk.begin, bk.end, ncclFloat16, false, d.stream));
        RBK_CUDA(cudaEventRecord(d.weights_ready[i], d.stream));
    }
    d.ag_pending = true;
    return RBK_OK;
}

// Order stream st after the FP16 all-gather of the bucket holding backward unit `unit`
// (-1: all buckets).  The forward calls it before each unit's first use of its weights.
int dp_wait_weights(rbk_model* m, int unit, cudaStream_t st) {
    DpState& d = m->dp;
    if (!d.on || !d.ag_pending) return RBK_OK;
    if (unit < 0) {
        for (cudaEvent_t e : d.weights_ready) RBK_CUDA(cudaStreamWaitEvent(st, e, 0));
        d.ag_pending = false;
        return RBK_OK;
    }
    RBK_CUDA(cudaStreamWaitEvent(st, d.weights_ready[d.unit_bucket[unit]], 0));
    if (unit == 0) d.ag_pending = false;           // the head is the forward's last unit
    return RBK_OK;
}

// All-gather the FP32 masters and both moments on st, so every rank holds all of them.
int dp_gather_state(rbk_model* m, cudaStream_t st) {
    DpState& d = m->dp;
    if (!d.on || !d.shard || !d.masters_partial) return RBK_OK;
    RBK_TRY(dp_wait_weights(m, -1, st));
    for (float* arena : {m->p32, m->m, m->v})
        for (const DpBucket& bk : d.plan) RBK_TRY(all_gather(m, arena, bk.begin, bk.end, ncclFloat32, true, st));
    d.masters_partial = false;
    return RBK_OK;
}

int dp_state_status(DpState& d);
int dp_status(rbk_model* m) { return dp_state_status(m->dp); }

// Create the communicators (non-blocking; a second one with a CTA cap when max_ctas > 0),
// the high-priority communication stream and the watchdog, on `device`.
int dp_open(DpState& d, int device, const void* id128, int rank, int world, int max_ctas, double timeout_in) {
    RBK_CUDA(cudaSetDevice(device));
    const double timeout_s = timeout_in > 0 ? timeout_in : 300.0;
    const double setup_s = std::max(timeout_s, kSetupBoundS);
    ncclUniqueId id;
    std::memcpy(&id, id128, sizeof(id));
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclComm_t comm = nullptr, tail = nullptr;
    ncclResult_t r = ncclCommInitRankConfig(&comm, world, id, rank, &cfg);
    if (r == ncclInProgress || r == ncclSuccess) r = settle(comm, setup_s);
    if (r != ncclSuccess) {
        set_error("ncclCommInitRankConfig failed: %s", r == ncclInProgress ? "timed out" : ncclGetErrorString(r));
        if (comm) ncclCommAbort(comm);
        return r == ncclInProgress ? RBK_ERR_TIMEOUT : RBK_ERR_NCCL;
    }
    if (max_ctas > 0) {
        // the capped communicator for the overlapped buckets; `comm` (uncapped) keeps the tail
        ncclConfig_t capped = NCCL_CONFIG_INITIALIZER;
        capped.blocking = 0;
        capped.maxCTAs = max_ctas;
        capped.minCTAs = 1;
        ncclComm_t c2 = nullptr;
        r = ncclCommSplit(comm, 0, rank, &c2, &capped);
        if (r == ncclInProgress || r == ncclSuccess) r = settle(comm, setup_s);
        if (r == ncclSuccess && c2) r = settle(c2, setup_s);
        if (r != ncclSuccess || !c2) {
            set_error("ncclCommSplit (capped communicator) failed: %s",
                      r == ncclInProgress ? "timed out" : ncclGetErrorString(r));
            if (c2) ncclCommAbort(c2);
            ncclCommAbort(comm);
            return r == ncclInProgress ? RBK_ERR_TIMEOUT : RBK_ERR_NCCL;
        }
        tail = comm;
        comm = c2;
    } else {
        tail = comm;
    }
    int lo = 0, hi = 0;
    RBK_CUDA(cudaDeviceGetStreamPriorityRange(&lo, &hi));
    RBK_CUDA(cudaStreamCreateWithPriority(&d.stream, cudaStreamNonBlocking, hi));
    RBK_CUDA(cudaEventCreateWithFlags(&d.all_done, cudaEventDisableTiming));
    d.rank = rank;
    d.world = world;
    d.max_ctas = max_ctas;
    d.watch = new DpWatch();
    d.watch->device = device;
    d.watch->timeout_s = timeout_s;
    d.watch->comms[0] = comm;
    d.watch->comms[1] = tail;
    d.watch->th = std::thread([w = d.watch] { w->loop(); });
    d.on = true;
    return RBK_OK;
}

// Drain, stop the watchdog and release the communicators and every event / buffer of d.
int dp_close(DpState& d) {
    if (!d.on) return RBK_OK;
    DpWatch* w = d.watch;
    // Wait for the collectives in flight; the watchdog keeps running meanwhile, so a hung one
    // is aborted after the timeout and this returns.
    cudaStreamSynchronize(d.stream);
    {
        std::lock_guard<std::mutex> lk(w->mu);
        w->stop = true;
    }
    w->th.join();
    if (w->comms[1] && w->comms[1] != w->comms[0]) ncclCommDestroy(w->comms[1]);
    if (w->comms[0]) ncclCommDestroy(w->comms[0]);
    for (cudaEvent_t e : w->all) cudaEventDestroy(e);
    delete w;
    for (auto& e : d.layer_done) cudaEventDestroy(e);
    cudaEventDestroy(d.all_done);
    for (auto& e : d.weights_ready) cudaEventDestroy(e);
    if (d.tail_done) cudaEventDestroy(d.tail_done);
    if (d.xbuf) cudaFree(d.xbuf);
    cudaStreamDestroy(d.stream);
    d = DpState();
    return RBK_OK;
}

int dp_state_status(DpState& d) {
    if (!d.on || !d.watch) return RBK_OK;
    std::lock_guard<std::mutex> lk(d.watch->mu);
    return d.watch->failed;
}

}  // namespace rbk

// Kernel-level data parallelism: the communicators, stream and watchdog of the model-level
// path without a model (the caller names the buffers).
struct rbk_dp {
    rbk::DpState d;
    cudaEvent_t ready = nullptr;
};

using namespace rbk;

extern "C" {

int rbk_dp_plan(const rbk_config* cfg, int64_t bucket_bytes, int64_t* out, int max, int* count) {
    RBK_REQUIRE(cfg && count && rbk_config_check(cfg) == 0 && bucket_bytes > 0, "rbk_dp_plan: bad arguments");
    const std::vector<DpBucket> p = dp_plan(cfg, std::max<int64_t>(bucket_bytes / 4, 1));
    *count = (int)p.size();
    for (int i = 0; i < (int)p.size() && i < max && out; ++i) {
        out[3 * i] = p[i].unit;
        out[3 * i + 1] = p[i].begin;
        out[3 * i + 2] = p[i].end;
    }
    return RBK_OK;
}

int rbk_dp_unique_id(void* id128) {
    RBK_REQUIRE(id128, "rbk_dp_unique_id: null pointer");
    static_assert(sizeof(ncclUniqueId) == RBK_NCCL_ID_BYTES, "NCCL unique id size");
    ncclResult_t r = ncclGetUniqueId(reinterpret_cast<ncclUniqueId*>(id128));
    if (r != ncclSuccess) {
        set_error("ncclGetUniqueId failed: %s", ncclGetErrorString(r));
        return RBK_ERR_NCCL;
    }
    return RBK_OK;
}

int rbk_model_dp_init_ex(rbk_model* m, const void* id128, int rank, int world, const rbk_dp_opts* o) {
    RBK_REQUIRE(m && id128 && o && world >= 1 && rank >= 0 && rank < world && o->bucket_bytes > 0,
                "rbk_model_dp_init_ex: bad arguments");
    RBK_REQUIRE(!m->dp.on, "rbk_model_dp_init_ex: already initialised");
    if (o->shard_optimizer) {
        for (const DpBucket& bk : dp_plan(&m->lay, std::max<int64_t>(o->bucket_bytes / 4, 1)))
            RBK_REQUIRE((bk.end - bk.begin) % (4 * (int64_t)world) == 0,
                        "rbk_model_dp_init_ex: the sharded optimizer needs every bucket to split into %d slices of a "
                        "multiple of 4 elements (bucket [%lld, %lld))", world, (long long)bk.begin, (long long)bk.end);
        RBK_REQUIRE(m->lora.rank == 0, "rbk_model_dp_init_ex: the sharded optimizer covers the base model, not LoRA");
    }
    RBK_TRY(dp_open(m->dp, m->ctx->device, id128, rank, world, o->max_ctas, o->timeout_s));
    DpState& d = m->dp;
    d.layer_done.resize(m->cfg.L + 2);
    for (auto& e : d.layer_done) RBK_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    d.bucket_elems = std::max<int64_t>(o->bucket_bytes / 4, 1);
    d.plan = dp_plan(&m->lay, d.bucket_elems);
    if (o->shard_optimizer) {
        d.shard = true;
        d.unit_bucket.assign(m->cfg.L + 2, 0);
        int first = 0;                                  // units first..bk.unit belong to bucket i
        for (int i = 0; i < (int)d.plan.size(); ++i) {
            const DpBucket& bk = d.plan[i];
            for (int u = first; u <= bk.unit; ++u) d.unit_bucket[u] = i;
            first = bk.unit + 1;
            d.own.push_back(bk.begin + (bk.end - bk.begin) / world * rank);
            d.own.push_back(bk.begin + (bk.end - bk.begin) / world * (rank + 1));
        }
        std::vector<int64_t> asc;                       // ascending address order
        for (int i = (int)d.own.size() - 2; i >= 0; i -= 2) {
            asc.push_back(d.own[i]);
            asc.push_back(d.own[i + 1]);
        }
        d.own = asc;
        RBK_CUDA(cudaMalloc(&d.xbuf, sizeof(float) * (2 + m->seg_off.size())));
        d.weights_ready.resize(d.plan.size());
        for (auto& e : d.weights_ready) RBK_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        RBK_CUDA(cudaEventCreateWithFlags(&d.tail_done, cudaEventDisableTiming));
    }
    return RBK_OK;
}

int rbk_model_dp_init(rbk_model* m, const void* id128, int rank, int world, int64_t bucket_bytes) {
    rbk_dp_opts o = {};
    o.bucket_bytes = bucket_bytes;
    o.max_ctas = (int)env_double("RBK_NCCL_MAX_CTAS", 0.0);
    o.timeout_s = env_double("RBK_NCCL_TIMEOUT_S", 300.0);
    o.shard_optimizer = (int)env_double("RBK_DP_SHARD", 0.0);
    return rbk_model_dp_init_ex(m, id128, rank, world, &o);
}

int rbk_model_dp_set_sync(rbk_model* m, int sync) {
    RBK_REQUIRE(m, "rbk_model_dp_set_sync: null model");
    m->dp.sync = sync != 0;
    return RBK_OK;
}

int rbk_model_dp_status(rbk_model* m) {
    RBK_REQUIRE(m, "rbk_model_dp_status: null model");
    const int s = dp_status(m);
    if (s != RBK_OK) set_error("data parallel: the communicator was aborted (%s)",
                               s == RBK_ERR_TIMEOUT ? "a collective timed out" : "an NCCL / CUDA error");
    return s;
}

int rbk_model_dp_shard_ranges(rbk_model* m, int64_t* out, int max, int* count) {
    RBK_REQUIRE(m && count, "rbk_model_dp_shard_ranges: bad arguments");
    const DpState& d = m->dp;
    *count = d.shard ? (int)d.own.size() / 2 : 0;
    for (int i = 0; i < *count && i < max && out; ++i) {
        out[2 * i] = d.own[2 * i];
        out[2 * i + 1] = d.own[2 * i + 1];
    }
    return RBK_OK;
}

int rbk_model_dp_gather_state(rbk_model* m, void* stream) {
    RBK_REQUIRE(m, "rbk_model_dp_gather_state: null model");
    if (m->dp.on) RBK_TRY(rbk_model_dp_status(m));
    return dp_gather_state(m, as_stream(stream));
}

int rbk_model_dp_abort(rbk_model* m) {
    RBK_REQUIRE(m, "rbk_model_dp_abort: null model");
    if (!m->dp.on || !m->dp.watch) return RBK_OK;
    std::lock_guard<std::mutex> lk(m->dp.watch->mu);
    m->dp.watch->abort_locked(RBK_ERR_NCCL);
    return RBK_OK;
}

int rbk_model_dp_shutdown(rbk_model* m) {
    RBK_REQUIRE(m, "rbk_model_dp_shutdown: null model");
    return dp_close(m->dp);
}

// ---------------------------------------------------------------- kernel level --
int rbk_dp_init(rbk_dp** out, int device, const void* id128, int rank, int world, const rbk_dp_opts* o) {
    RBK_REQUIRE(out && id128 && world >= 1 && rank >= 0 && rank < world, "rbk_dp_init: bad arguments");
    *out = nullptr;
    rbk_dp* p = new rbk_dp();
    int st = dp_open(p->d, device, id128, rank, world, o ? o->max_ctas : 0, o ? o->timeout_s : 0.0);
    if (st == RBK_OK && cudaEventCreateWithFlags(&p->ready, cudaEventDisableTiming) != cudaSuccess) {
        set_error("rbk_dp_init: cudaEventCreate failed");
        dp_close(p->d);
        st = RBK_ERR_CUDA;
    }
    if (st != RBK_OK) {
        delete p;
        return st;
    }
    *out = p;
    return RBK_OK;
}

int rbk_dp_bucket_ready(rbk_dp* dp, float* buf, int64_t n, void* stream) {
    RBK_REQUIRE(dp && dp->d.on && buf && n > 0, "rbk_dp_bucket_ready: bad arguments");
    RBK_TRY(rbk_dp_status(dp));
    RBK_CUDA(cudaEventRecord(dp->ready, as_stream(stream)));
    RBK_CUDA(cudaStreamWaitEvent(dp->d.stream, dp->ready, 0));
    return allreduce(dp->d, buf, (size_t)n, false);
}

int rbk_dp_finish(rbk_dp* dp, void* stream) {
    RBK_REQUIRE(dp && dp->d.on, "rbk_dp_finish: bad arguments");
    RBK_TRY(rbk_dp_status(dp));
    RBK_CUDA(cudaEventRecord(dp->d.all_done, dp->d.stream));
    RBK_CUDA(cudaStreamWaitEvent(as_stream(stream), dp->d.all_done, 0));
    return RBK_OK;
}

int rbk_dp_status(rbk_dp* dp) {
    RBK_REQUIRE(dp, "rbk_dp_status: null handle");
    const int s = dp_state_status(dp->d);
    if (s != RBK_OK) set_error("data parallel: the communicator was aborted (%s)",
                               s == RBK_ERR_TIMEOUT ? "a collective timed out" : "an NCCL / CUDA error");
    return s;
}

int rbk_dp_abort(rbk_dp* dp) {
    RBK_REQUIRE(dp, "rbk_dp_abort: null handle");
    if (!dp->d.on || !dp->d.watch) return RBK_OK;
    std::lock_guard<std::mutex> lk(dp->d.watch->mu);
    dp->d.watch->abort_locked(RBK_ERR_NCCL);
    return RBK_OK;
}

int rbk_dp_destroy(rbk_dp* dp) {
    if (!dp) return RBK_OK;
    const int st = dp_close(dp->d);
    if (dp->ready) cudaEventDestroy(dp->ready);
    delete dp;
    return st;
}

}  // extern "C"
