// wb_prof.cu -- CUDA-event timing of named kernels (wb_context_profile).
#include "wb_internal.h"

#include <map>
#include <string>
#include <vector>

namespace wb {

struct Profiler {
    std::string filter;  // "" = every named kernel, else only names containing it
    struct Rec {
        const char *name;
        cudaEvent_t a, b;
    };
    std::vector<Rec> recs;
    std::vector<cudaEvent_t> pool;
    const char *open_name = nullptr;
    cudaEvent_t open_ev = nullptr;
    cudaEvent_t get() {
        if (!pool.empty()) {
            cudaEvent_t e = pool.back();
            pool.pop_back();
            return e;
        }
        cudaEvent_t e = nullptr;
        cudaEventCreate(&e);
        return e;
    }
};

Profiler *&prof_current() {
    static thread_local Profiler *p = nullptr;
    return p;
}

// Inside stream capture a plain record only orders the capture; an event
// record node (timed at every replay of the graph) needs the external flag.
static void record(cudaEvent_t e, cudaStream_t st) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &cs) == cudaSuccess && cs == cudaStreamCaptureStatusActive)
        cudaEventRecordWithFlags(e, st, cudaEventRecordExternal);
    else
        cudaEventRecord(e, st);
}

void prof_begin(const char *name, cudaStream_t st) {
    Profiler *p = prof_current();
    if (!p || (!p->filter.empty() && std::string(name).find(p->filter) == std::string::npos)) return;
    p->open_name = name;
    p->open_ev = p->get();
    record(p->open_ev, st);
}

void prof_end(cudaStream_t st) {
    Profiler *p = prof_current();
    if (!p || !p->open_name) return;
    cudaEvent_t b = p->get();
    record(b, st);
    p->recs.push_back({p->open_name, p->open_ev, b});
    p->open_name = nullptr;
}

Profiler *prof_create(const char *filter) {
    Profiler *p = new Profiler();
    p->filter = filter ? filter : "";
    return p;
}

void prof_destroy(Profiler *p) {
    if (!p) return;
    for (auto &r : p->recs) {
        cudaEventDestroy(r.a);
        cudaEventDestroy(r.b);
    }
    for (auto e : p->pool) cudaEventDestroy(e);
    delete p;
}

// Resolve all recorded pairs (the caller synchronised the stream) into
// "name<TAB>launches<TAB>total_ms" lines; recycles the events.
std::string prof_report(Profiler *p) {
    std::map<std::string, std::pair<long, double>> agg;
    for (auto &r : p->recs) {
        float ms = 0.0f;
        if (cudaEventElapsedTime(&ms, r.a, r.b) != cudaSuccess) {
            cudaGetLastError();
            ms = 0.0f;
        }
        auto &e = agg[r.name];
        e.first += 1;
        e.second += ms;
        p->pool.push_back(r.a);
        p->pool.push_back(r.b);
    }
    p->recs.clear();
    std::string out;
    for (auto &kv : agg)
        out += kv.first + "\t" + std::to_string(kv.second.first) + "\t" + std::to_string(kv.second.second) + "\n";
    return out;
}

}  // namespace wb
