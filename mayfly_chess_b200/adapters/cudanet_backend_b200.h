// The C++ search's two network interfaces on libcudanet_b200.so: mayfly2::Net (mayfly/chess/cpp/search2.h:55-88,
// the persistent tree) and mayfly::NetBackend (cpp/netbackend.h:43-48). A drop-in for the reference's
// cudanet/cudanet_backend.h: the same three factory functions (make_cuda_net, cuda_net_fingerprint,
// make_cuda_backend) with the same meaning, so cpp/pyext.cpp:195-203 builds unchanged against this header. Put the
// reference's cpp/ folder and this repository's include/ on the include path and link libcudanet_b200.so.
// Header-only.
//
// mayfly2::CudaB200Net (cudanet_backend.cpp:42-102 CudaNetAdapter):
//   evaluate       cudanet_evaluate: the batch search2 encoded (Batch: ids, cast, hm, ep, I, M), the policy
//                  logits cut to each row's legal moves, the value and the per-move q back (Out), which is
//                  exactly what search2 expects (the reference adapter passes them through the same way)
//   submit/collect Settings::pipeline's halves: cudanet_begin copies the batch into pinned staging and queues
//                  the pass, so `in` may go once submit returns; cudanet_end waits for the oldest batch. At most
//                  two in flight, as search2 keeps them.
// Errors come back from the library as -1 with a message and are thrown as std::runtime_error, as search2's
// Net contract asks ("throws on failure").
// mayfly::CudaB200Backend (cudanet_backend.cpp:105-151 CudaBackend): the same pass, then the cut policy scattered
// into full B x 4162 rows at each row's legal moves (policy[b*4162 + I[b*wide+j]], j < widths[b]), every other
// entry 0 — all the search reads, as the reference's CUDA backend documents (cudanet_backend.h:25-30).
#pragma once
#include <deque>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "cudanet_b200.h"
#include "netbackend.h"
#include "search2.h"

namespace mayfly2 {

class CudaB200Net : public Net {
public:
    CudaB200Net(const std::string& weights_path, int device)
    {
        char err[1024] = {0};
        h_ = cudanet_create(weights_path.c_str(), device, err, sizeof err);
        if (!h_) throw std::runtime_error(std::string("cudanet_create: ") + err);
    }
    ~CudaB200Net() override { cudanet_destroy(h_); }
    CudaB200Net(const CudaB200Net&) = delete;
    CudaB200Net& operator=(const CudaB200Net&) = delete;

    void evaluate(const Batch& in, Out& out) override
    {
        check(in);
        size_out(out, in.B, in.wide);
        char err[1024] = {0};
        if (cudanet_evaluate(h_, in.B, in.wide, in.ids.data(), in.cast.data(), in.hm.data(), in.ep.data(),
                             in.I.data(), in.M.data(), out.pol.data(), out.val.data(), out.qv.data(), err,
                             sizeof err))
            throw std::runtime_error(std::string("cudanet_evaluate: ") + err);
    }

    void submit(const Batch& in) override
    {
        check(in);
        char err[1024] = {0};
        if (cudanet_begin(h_, in.B, in.wide, in.ids.data(), in.cast.data(), in.hm.data(), in.ep.data(),
                          in.I.data(), in.M.data(), err, sizeof err))
            throw std::runtime_error(std::string("cudanet_begin: ") + err);
        fly_.emplace_back(in.B, in.wide);
    }

    void collect(Out& out) override
    {
        if (fly_.empty()) throw std::runtime_error("cudanet_b200: collect with no batch on the card");
        const std::pair<int, int> f = fly_.front();
        fly_.pop_front();
        size_out(out, f.first, f.second);
        char err[1024] = {0};
        if (cudanet_end(h_, out.pol.data(), out.val.data(), out.qv.data(), err, sizeof err))
            throw std::runtime_error(std::string("cudanet_end: ") + err);
    }

    int max_batch() const { return cudanet_max_batch(h_); }
    std::string fingerprint() const
    {
        char buf[256] = {0};
        return cudanet_fingerprint(h_, buf, sizeof buf) < 0 ? std::string() : std::string(buf);
    }

private:
    // search2's Batch holds its arrays as vectors; their sizes must match B and wide (the reference adapter's
    // check_batch, cudanet_backend.cpp:27-37)
    static void check(const Batch& in)
    {
        if (in.B < 1 || in.wide < 1) throw std::runtime_error("cudanet_b200: empty batch");
        const size_t b = static_cast<size_t>(in.B), w = static_cast<size_t>(in.wide);
        if (in.ids.size() != b * 64 || in.cast.size() != b * 4 || in.hm.size() != b || in.ep.size() != b ||
            in.I.size() != b * w || in.M.size() != b * w)
            throw std::runtime_error("cudanet_b200: batch arrays have the wrong sizes");
    }
    static void size_out(Out& out, int B, int wide)
    {
        const size_t b = static_cast<size_t>(B), w = static_cast<size_t>(wide);
        out.pol.resize(b * w);
        out.val.resize(b);
        out.qv.resize(b * w);
    }

    void* h_ = nullptr;
    std::deque<std::pair<int, int>> fly_;   // (B, wide) of each batch submitted and not yet collected
};

// cudanet_backend.h:13-17: the evaluator on `device` from a .cnw file, behind mayfly2::Net
inline Net* make_cuda_net(const std::string& weights_path, int device)
{
    return new CudaB200Net(weights_path, device);
}

// cudanet_backend.h:19-21: the weight file's fingerprint for a Net made above, empty for any other Net
inline std::string cuda_net_fingerprint(Net* net)
{
    CudaB200Net* a = dynamic_cast<CudaB200Net*>(net);
    return a ? a->fingerprint() : std::string();
}

}  // namespace mayfly2

namespace mayfly {

class CudaB200Backend : public NetBackend {
public:
    CudaB200Backend(const std::string& weights_path, int device) : net_(weights_path, device) {}

    void evaluate(const NetBatch& in, NetResult& out) override
    {
        if (in.widths.size() != static_cast<size_t>(in.B))
            throw std::runtime_error("cudanet_b200: widths has the wrong size");
        mayfly2::Batch b;
        b.B = in.B;
        b.wide = in.wide;
        b.ids = in.ids;
        b.cast = in.cast;
        b.hm = in.hm;
        b.ep = in.ep;
        b.I = in.I;
        b.M = in.M;
        mayfly2::Out o;
        net_.evaluate(b, o);
        const size_t B = static_cast<size_t>(in.B), W = static_cast<size_t>(in.wide);
        out.val = std::move(o.val);
        out.qv = std::move(o.qv);
        out.policy.assign(B * static_cast<size_t>(kMoves), 0.0f);
        for (size_t r = 0; r < B; ++r) {
            const size_t n = static_cast<size_t>(in.widths[r]);
            if (n > W) throw std::runtime_error("cudanet_b200: a row is wider than wide");
            float* row = out.policy.data() + r * static_cast<size_t>(kMoves);
            for (size_t j = 0; j < n; ++j) {
                const int64_t m = in.I[r * W + j];
                if (m < 0 || m >= kMoves) throw std::runtime_error("cudanet_b200: a move index is out of range");
                row[m] = o.pol[r * W + j];
            }
        }
    }

private:
    mayfly2::CudaB200Net net_;
};

// cudanet_backend.h:23-31
inline NetBackend* make_cuda_backend(const std::string& weights_path, int device)
{
    return new CudaB200Backend(weights_path, device);
}

}  // namespace mayfly
