// exl3b_cepf.cu -- copy-engine expert prefetch (reference: moe_prefetch_plan and the PfWorker host thread,
// kernels/moe-a8/exl3_moe.a8.sycl:1048-1142, and the plan / commit modes of launch_ensure, :838-905, 1010-1036).
//
// The experts predicted for a layer get LRU slots from a plan kernel on the compute stream; their blobs are copied by
// the copy engine, driven by a host thread, so no SM time goes to the copies and the compute stream never waits:
//   plan   (compute stream): commit what has landed; if this layer's previous plan is still in flight, do nothing;
//          else claim slots exactly as moe_prefetch does (tick not advanced), PIN them (slot_last = INT_MAX: never a
//          victim, and a hit keeps the pin), record them in pend[layer] and publish them to the pinned host plan
//          buffer, its sequence number last behind a system-scope fence;
//   worker (host thread): a new sequence number in a layer's plan -> one cudaMemcpyAsync per (expert, slot) on the
//          copy stream, then a one-thread kernel on that stream writes done_seq[layer] = seq.  The value travels in
//          the launch, so the copy engine never reads a host word the worker may rewrite for a later plan;
//   commit (compute stream, before every cached MoE call and inside every plan): each layer whose done_seq reached
//          its pending seq gets its table entries pointed at the slots and the slots unpinned (slot_last = the tick
//          of the plan).
// Until its commit a planned expert's table entry stays at its host copy, so every read before the commit is a
// correct zero-copy read, and its slot is written by the copy engine alone.
//
// pend (device, per layer kPendStride int32): [n, seq, T, (expert, slot) x kPendMax]; n = 0: nothing in flight.
// plan buffer (pinned host, per layer 4 + 2E int32): [seq, n, T, layer, (expert, slot) x n].
#include <atomic>
#include <memory>
#include <mutex>
#include <thread>
#include <vector>

#include "exl3b_common.cuh"
#include "exl3b_capi_util.h"
#include "exl3b_ensure.cuh"

namespace exl3b {

constexpr int kPendStride = 35;
constexpr int kPendMax = 16;
constexpr int kPinned = 0x7FFFFFFF;

struct CommitArgs {
    int32_t* pend; const int32_t* done_seq; int n_layers; int E; int S;
    int64_t* ptrs_all; int32_t* slot_last; int64_t slot_base; int64_t blob;
};

// One thread per layer: a landed plan (done_seq >= its seq) is committed and cleared.
__device__ __forceinline__ void commit_landed(const CommitArgs& c) {
    for (int li = threadIdx.x; li < c.n_layers; li += blockDim.x) {
        int32_t* pl = c.pend + (int64_t)li * kPendStride;
        const int n = pl[0];
        if (n <= 0) continue;
        const int done = *reinterpret_cast<volatile const int32_t*>(c.done_seq + li);
        if (done < pl[1]) continue;
        if (n > kPendMax) { set_error(kErrBounds); pl[0] = 0; continue; }
        for (int i = 0; i < n; ++i) {
            const int e = pl[3 + 2 * i], s = pl[4 + 2 * i];
            if (e < 0 || e >= c.E || s < 0 || s >= c.S) { set_error(kErrBounds); continue; }
            c.ptrs_all[(int64_t)li * c.E + e] = c.slot_base + (int64_t)s * c.blob;
            c.slot_last[s] = pl[2];
        }
        pl[0] = 0;
    }
}

__global__ void __launch_bounds__(64) cepf_commit_kernel(CommitArgs c) { commit_landed(c); }

struct PlanArgs {
    int32_t* plan;        // this layer's record in the pinned host plan buffer
    int32_t* plan_seq;    // device [n_layers]
};

__global__ void __launch_bounds__(kEnsureThreads) cepf_plan_kernel(EnsureArgs a, CommitArgs c, PlanArgs p) {
    commit_landed(c);
    __syncthreads();
    int32_t* pl = c.pend + (int64_t)a.layer * kPendStride;
    if (pl[0] > 0) {   // the previous plan of this layer is still in flight: this prediction is dropped
        if (threadIdx.x == 0) a.fill_list[0] = 0;
        return;
    }
    ensure_block(a);   // prefetch mode: fill_list = [n, expert...], pf_slot = [slot...], tick unchanged
    __syncthreads();
    const int n = min(a.fill_list[0], kPendMax);
    const int T = a.tick[0];
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int e = a.fill_list[1 + i], s = a.pf_slot[i];
        a.slot_last[s] = kPinned;
        pl[3 + 2 * i] = e;
        pl[4 + 2 * i] = s;
        p.plan[4 + 2 * i] = e;
        p.plan[5 + 2 * i] = s;
        __threadfence_system();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        p.plan[1] = n;
        p.plan[2] = T;
        p.plan[3] = a.layer;
        const int seq = p.plan_seq[a.layer] + 1;
        p.plan_seq[a.layer] = seq;
        if (n > 0) { pl[1] = seq; pl[2] = T; pl[0] = n; }
        __threadfence_system();   // the pairs and the header reach host memory before the sequence number
        *reinterpret_cast<volatile int32_t*>(p.plan) = seq;
    }
}

__global__ void cepf_done_kernel(int32_t* done, int seq) { *reinterpret_cast<volatile int32_t*>(done) = seq; }

// The host side: polls the plan buffer, turns each new plan into copy-engine copies and the done write.
struct CepfWorker {
    const int32_t* plans = nullptr;
    int L = 0, E = 0, S = 0, device = 0;
    std::vector<int64_t> host_base;
    int64_t slot_base = 0, blob = 0, hstride = 0;
    int32_t* done_seq = nullptr;
    cudaStream_t stream = nullptr;
    std::vector<int> seen;
    std::atomic<bool> stop{false};
    std::atomic<long long> n_plans{0}, n_copies{0};
    std::atomic<int> error{0};
    std::thread th;

    bool scan() {
        bool any = false;
        for (int li = 0; li < L; ++li) {
            const int32_t* rec = plans + (int64_t)li * (4 + 2 * E);
            const int seq = __atomic_load_n(rec, __ATOMIC_ACQUIRE);
            if (seq == seen[li]) continue;
            seen[li] = seq;
            any = true;
            // the device writes the pairs, then n, then seq, each behind a system-scope fence; a record is rewritten
            // only after its plan committed (which needs this worker's done write), so reading n and then the pairs
            // in order sees one plan: at worst a newer one under an older seq, whose copies are right and whose done
            // value (the older seq) commits nothing
            const int n = __atomic_load_n(rec + 1, __ATOMIC_ACQUIRE);
            bool ok = n >= 0 && n <= kPendMax;
            for (int i = 0; ok && i < n; ++i) {
                const int e = __atomic_load_n(rec + 4 + 2 * i, __ATOMIC_RELAXED);
                const int s = __atomic_load_n(rec + 5 + 2 * i, __ATOMIC_RELAXED);
                if (e < 0 || e >= E || s < 0 || s >= S) { ok = false; break; }
                ok = cudaMemcpyAsync(reinterpret_cast<void*>(slot_base + (int64_t)s * blob),
                                     reinterpret_cast<const void*>(host_base[li] + (int64_t)e * hstride), (size_t)blob,
                                     cudaMemcpyDefault, stream) == cudaSuccess;
            }
            if (ok && n > 0) {
                cepf_done_kernel<<<1, 1, 0, stream>>>(done_seq + li, seq);
                ok = cudaGetLastError() == cudaSuccess;
            }
            if (!ok) {   // no done write: the plan stays in flight and its experts are read from host
                int expect = 0;
                error.compare_exchange_strong(expect, EXL3B_ECUDA);
                continue;
            }
            n_plans++;
            n_copies += n;
        }
        return any;
    }

    void run() {
        if (cudaSetDevice(device) != cudaSuccess) { error = EXL3B_ECUDA; return; }
        while (!stop.load(std::memory_order_acquire))
            if (!scan()) std::this_thread::yield();
        scan();   // plans published before the stop
        if (cudaStreamSynchronize(stream) != cudaSuccess) {
            int expect = 0;
            error.compare_exchange_strong(expect, EXL3B_ECUDA);
        }
    }
};

// Owned by start / stop only (no static destructor: a joinable thread destroyed at exit would end the process).
std::mutex g_cepf_mutex;
CepfWorker* g_cepf = nullptr;

}  // namespace exl3b

using namespace exl3b;

extern "C" EXL3B_API int exl3b_cepf_commit(int32_t* pend, const int32_t* done_seq, int n_layers, int E, int S,
                                           int64_t* ptrs_all, int32_t* slot_last, int64_t slot_base, int64_t blob,
                                           void* stream) {
    EXL3B_CHECK(pend && done_seq && ptrs_all && slot_last, "exl3b_cepf_commit: null pointer");
    EXL3B_CHECK(n_layers >= 0 && E >= 1 && S >= 0, "exl3b_cepf_commit: bad sizes");
    if (n_layers == 0 || S == 0) return 0;
    CommitArgs c{pend, done_seq, n_layers, E, S, ptrs_all, slot_last, slot_base, blob};
    cepf_commit_kernel<<<1, 64, 0, (cudaStream_t)stream>>>(c);
    return exl3b_launch_status("exl3b_cepf_commit");
}

extern "C" EXL3B_API int exl3b_cepf_plan(const int32_t* ids, int n, int layer, int E, int S, int64_t* ptrs_all,
                                         int32_t* slot_of, int32_t* slot_key, int32_t* slot_last, int32_t* tick,
                                         const int64_t* host_base, int64_t slot_base, int64_t blob, int64_t hstride,
                                         int32_t* pf_list, int32_t* pf_slot, int max_fill, int32_t* plans,
                                         int32_t* plan_seq, int32_t* pend, const int32_t* done_seq, int n_layers,
                                         void* stream) {
    EXL3B_CHECK(E >= 1 && E <= 1024 && n >= 0 && S >= 0, "exl3b_cepf_plan: bad sizes");
    EXL3B_CHECK(layer >= 0 && layer < n_layers, "exl3b_cepf_plan: layer outside the plan buffer");
    EXL3B_CHECK(ids && ptrs_all && slot_of && tick && host_base && pf_list && pf_slot && plans && plan_seq && pend &&
                done_seq, "exl3b_cepf_plan: null pointer");
    EXL3B_CHECK(S == 0 || (slot_key && slot_last), "exl3b_cepf_plan: slot tables missing");
    EXL3B_CHECK(max_fill >= 0 && max_fill <= kPendMax, "exl3b_cepf_plan: 0 <= max_fill <= 16");
    if (S == 0 || n == 0) return 0;
    EnsureArgs a{const_cast<int32_t*>(ids), nullptr, n, layer, E, S, ptrs_all, slot_of, slot_key, slot_last, tick,
                 host_base, slot_base, blob, hstride > 0 ? hstride : blob, nullptr, pf_list, max_fill, 1, pf_slot,
                 nullptr, nullptr, 0, nullptr, nullptr};
    CommitArgs c{pend, done_seq, n_layers, E, S, ptrs_all, slot_last, slot_base, blob};
    PlanArgs p{plans + (int64_t)layer * (4 + 2 * E), plan_seq};
    cepf_plan_kernel<<<1, kEnsureThreads, 0, (cudaStream_t)stream>>>(a, c, p);
    return exl3b_launch_status("exl3b_cepf_plan");
}

extern "C" EXL3B_API int exl3b_cepf_worker_start(const int32_t* plans, int n_layers, int E, int S,
                                                 const int64_t* host_base, int64_t slot_base, int64_t blob,
                                                 int64_t hstride, int32_t* done_seq, int device, void* copy_stream) {
    EXL3B_CHECK(plans && host_base && done_seq, "exl3b_cepf_worker_start: null pointer");
    EXL3B_CHECK(n_layers >= 1 && E >= 1 && S >= 0 && blob > 0, "exl3b_cepf_worker_start: bad sizes");
    std::lock_guard<std::mutex> lock(g_cepf_mutex);
    if (g_cepf) return exl3b_fail(EXL3B_EINVAL, "exl3b_cepf_worker_start: the worker is already running");
    auto w = std::make_unique<CepfWorker>();
    w->plans = plans;
    w->L = n_layers;
    w->E = E;
    w->S = S;
    w->device = device;
    w->host_base.assign(host_base, host_base + n_layers);
    w->slot_base = slot_base;
    w->blob = blob;
    w->hstride = hstride > 0 ? hstride : blob;
    w->done_seq = done_seq;
    w->stream = (cudaStream_t)copy_stream;
    w->seen.resize(n_layers);
    for (int li = 0; li < n_layers; ++li) w->seen[li] = __atomic_load_n(plans + (int64_t)li * (4 + 2 * E), __ATOMIC_ACQUIRE);
    CepfWorker* raw = w.release();
    raw->th = std::thread([raw] { raw->run(); });
    g_cepf = raw;
    return 0;
}

extern "C" EXL3B_API int exl3b_cepf_worker_stop(int64_t* counts) {
    std::unique_ptr<CepfWorker> w;
    {
        std::lock_guard<std::mutex> lock(g_cepf_mutex);
        w.reset(g_cepf);
        g_cepf = nullptr;
    }
    if (counts) counts[0] = counts[1] = 0;
    if (!w) return 0;
    w->stop.store(true, std::memory_order_release);
    w->th.join();
    if (counts) {
        counts[0] = w->n_plans.load();
        counts[1] = w->n_copies.load();
    }
    if (w->error.load()) return exl3b_fail(w->error.load(), "exl3b_cepf_worker: a copy or its done write failed");
    return 0;
}

extern "C" EXL3B_API int exl3b_cepf_worker_running() {
    std::lock_guard<std::mutex> lock(g_cepf_mutex);
    return g_cepf != nullptr;
}
