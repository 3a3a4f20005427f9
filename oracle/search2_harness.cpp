// TEST INFRASTRUCTURE ONLY. The reference's own C++ search (mayfly/chess/cpp/search2.{h,cpp}, compiled from its
// sources by oracle/Makefile into oracle/_ref/libsearch2_b200.so together with chess_core.cpp) driving this
// repository's evaluator through the product adapter mayfly_chess_b200/adapters/cudanet_backend_b200.h. A flat C
// interface for tests/test_search2_gpu.py:
//
//   s2_open     a CudaB200Net on a weight file, wrapped in a recorder that can keep every batch search2 sends and
//               what came back. mode 0: the pipeline's submit/collect go to the adapter (cudanet_begin/end);
//               mode 1: the recorder leaves submit/collect to mayfly2::Net's defaults (keep a copy, evaluate on
//               collect), which search2.h:72-75 states gives the same numbers.
//   s2_search   one search from a FEN on a fresh tree: search2's Settings defaults with the given batch and
//               pipeline, expand_root when needed, step() until the root has `target` visits or the tree is
//               saturated, finish(); the root's moves, visit counts, choose() and the tree's counters out.
//   s2_record / s2_recorded / s2_get   the recorded batches and outputs.
//   s2_backend  one batch through mayfly::NetBackend (make_cuda_backend): full policy rows, val, qv.
#include <cstdint>
#include <cstring>
#include <deque>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "../mayfly_chess_b200/adapters/cudanet_backend_b200.h"

namespace {

struct Record {
    mayfly2::Batch in;
    mayfly2::Out out;
};

class Recorder : public mayfly2::Net {
public:
    Recorder(mayfly2::Net* inner, bool forward_pipeline) : inner_(inner), fwd_(forward_pipeline) {}
    void evaluate(const mayfly2::Batch& in, mayfly2::Out& out) override
    {
        inner_->evaluate(in, out);
        if (on) rec.push_back(Record{in, out});
    }
    void submit(const mayfly2::Batch& in) override
    {
        if (!fwd_) {
            mayfly2::Net::submit(in);
            return;
        }
        inner_->submit(in);
        pend_.push_back(in);
    }
    void collect(mayfly2::Out& out) override
    {
        if (!fwd_) {
            mayfly2::Net::collect(out);
            return;
        }
        inner_->collect(out);
        if (pend_.empty()) throw std::runtime_error("recorder: collect with nothing submitted");
        if (on) rec.push_back(Record{pend_.front(), out});
        pend_.pop_front();
    }
    bool on = false;
    std::vector<Record> rec;

private:
    mayfly2::Net* inner_;
    bool fwd_;
    std::deque<mayfly2::Batch> pend_;
};

struct Handle {
    std::unique_ptr<mayfly2::Net> net;
    std::unique_ptr<Recorder> rec;
    std::unique_ptr<mayfly::NetBackend> backend;
    std::string weights;
    int device = 0;
};

void put(char* err, int len, const char* msg)
{
    if (err && len > 0) {
        std::strncpy(err, msg, (size_t)len - 1);
        err[len - 1] = 0;
    }
}

}  // namespace

extern "C" {

void* s2_open(const char* weights, int device, int mode, char* err, int err_len)
{
    try {
        auto h = std::make_unique<Handle>();
        h->net.reset(mayfly2::make_cuda_net(weights, device));
        if (mayfly2::cuda_net_fingerprint(h->net.get()).empty()) throw std::runtime_error("no fingerprint");
        h->rec = std::make_unique<Recorder>(h->net.get(), mode == 0);
        h->weights = weights;
        h->device = device;
        return h.release();
    } catch (const std::exception& e) {
        put(err, err_len, e.what());
        return nullptr;
    }
}

void s2_close(void* hp) { delete static_cast<Handle*>(hp); }

void s2_record(void* hp, int on)
{
    Handle* h = static_cast<Handle*>(hp);
    h->rec->on = on != 0;
    if (on) h->rec->rec.clear();
}

int s2_recorded(void* hp) { return (int)static_cast<Handle*>(hp)->rec->rec.size(); }

// Batch i: its B and wide always; the arrays when the pointers are not null (the caller sized them from a first
// call with nulls). Returns 0, or -1 for a bad index.
int s2_get(void* hp, int i, int* B, int* wide, int64_t* ids, float* cast, int64_t* hm, int64_t* ep, int64_t* I,
           uint8_t* M, float* pol, float* val, float* qv)
{
    Handle* h = static_cast<Handle*>(hp);
    if (i < 0 || i >= (int)h->rec->rec.size()) return -1;
    const Record& r = h->rec->rec[(size_t)i];
    *B = r.in.B;
    *wide = r.in.wide;
    if (!ids) return 0;
    std::memcpy(ids, r.in.ids.data(), 8 * r.in.ids.size());
    std::memcpy(cast, r.in.cast.data(), 4 * r.in.cast.size());
    std::memcpy(hm, r.in.hm.data(), 8 * r.in.hm.size());
    std::memcpy(ep, r.in.ep.data(), 8 * r.in.ep.size());
    std::memcpy(I, r.in.I.data(), 8 * r.in.I.size());
    std::memcpy(M, r.in.M.data(), r.in.M.size());
    std::memcpy(pol, r.out.pol.data(), 4 * r.out.pol.size());
    std::memcpy(val, r.out.val.data(), 4 * r.out.val.size());
    std::memcpy(qv, r.out.qv.data(), 4 * r.out.qv.size());
    return 0;
}

// stats: evals, batches, cache_hits, collisions, tree nodes, then (Settings::prof, search2.h:118-126) the
// microseconds of all steps, of the network inside them (evaluate, or submit + collect with the pipeline) and of
// the batch encoding (MCTS._prepare). Returns the root's move count, or -1 with err.
int s2_search(void* hp, const char* fen, int batch, int pipeline, double target, int* moves, float* N, int cap,
              int* chosen, long long* stats, char* err, int err_len)
{
    try {
        Handle* h = static_cast<Handle*>(hp);
        mayfly::init_tables();
        mayfly::Pos p;
        if (!mayfly::parse_fen(fen, p)) throw std::runtime_error("bad FEN");
        mayfly2::Settings s;
        s.batch = batch;
        s.pipeline = pipeline;
        s.prof = true;
        mayfly2::Tree t(h->rec.get(), s);
        t.begin(p, std::vector<mayfly::Pos>(), false);
        if (t.needs_eval()) t.expand_root();
        for (int guard = 0; t.root()->sum_n < target && guard < 1000000; ++guard)
            if (t.step(target, -1.0) == 2) break;
        t.finish();
        mayfly2::Node* r = t.root();
        const int n = (int)r->moves.size();
        for (int k = 0; k < n && k < cap; ++k) {
            moves[k] = r->moves[(size_t)k];
            N[k] = r->N.empty() ? 0.0f : r->N[(size_t)k];
        }
        *chosen = t.choose();
        const mayfly2::Stats& st = t.stats();
        stats[0] = st.evals;
        stats[1] = st.batches;
        stats[2] = st.cache_hits;
        stats[3] = st.collisions;
        stats[4] = t.tree_nodes();
        const mayfly2::Prof& pf = t.prof();
        stats[5] = (long long)(1e6 * pf.step);
        stats[6] = (long long)(1e6 * (pf.net + pf.submit + pf.collect));
        stats[7] = (long long)(1e6 * pf.encode);
        return n;
    } catch (const std::exception& e) {
        put(err, err_len, e.what());
        return -1;
    }
}

// policy: B x 4162 f32, val: B, qv: B x wide. Returns 0, or -1 with err.
int s2_backend(void* hp, int B, int wide, const int64_t* ids, const float* cast, const int64_t* hm,
               const int64_t* ep, const int64_t* I, const uint8_t* M, const int* widths, float* policy, float* val,
               float* qv, char* err, int err_len)
{
    try {
        Handle* h = static_cast<Handle*>(hp);
        if (!h->backend) h->backend.reset(mayfly::make_cuda_backend(h->weights, h->device));
        mayfly::NetBatch in;
        const size_t b = (size_t)B, w = (size_t)wide;
        in.B = B;
        in.wide = wide;
        in.ids.assign(ids, ids + b * 64);
        in.cast.assign(cast, cast + b * 4);
        in.hm.assign(hm, hm + b);
        in.ep.assign(ep, ep + b);
        in.I.assign(I, I + b * w);
        in.M.assign(M, M + b * w);
        in.widths.assign(widths, widths + b);
        mayfly::NetResult out;
        h->backend->evaluate(in, out);
        std::memcpy(policy, out.policy.data(), 4 * out.policy.size());
        std::memcpy(val, out.val.data(), 4 * out.val.size());
        std::memcpy(qv, out.qv.data(), 4 * out.qv.size());
        return 0;
    } catch (const std::exception& e) {
        put(err, err_len, e.what());
        return -1;
    }
}

}  // extern "C"
