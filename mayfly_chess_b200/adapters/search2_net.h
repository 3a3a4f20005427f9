// mayfly2::Net (the reference's C++ search, mayfly/chess/cpp/search2.h:55-88) on libcudanet_b200.so.
//
// The reference builds its search extension with its own CUDA backend behind this interface
// (mayfly/chess/cudanet/cudanet_backend.cpp:42-102 CudaNetAdapter, chosen by cpp/pyext.cpp:195-203 for ".cnw"
// paths). This is the same adapter over this library's C ABI: include it after search2.h, with include/ of this
// repository on the include path, and link libcudanet_b200.so. Header-only.
//
//   evaluate       cudanet_evaluate: the batch search2 encoded (Batch: ids, cast, hm, ep, I, M), the policy
//                  logits cut to each row's legal moves, the value and the per-move q back (Out), which is
//                  exactly what search2 expects (the reference adapter passes them through the same way)
//   submit/collect Settings::pipeline's halves: cudanet_begin copies the batch into pinned staging and queues
//                  the pass, so `in` may go once submit returns; cudanet_end waits for the oldest batch. At most
//                  two in flight, as search2 keeps them.
// Errors come back from the library as -1 with a message and are thrown as std::runtime_error, as search2's
// Net contract asks ("throws on failure").
#pragma once
#include <deque>
#include <stdexcept>
#include <string>
#include <utility>

#include "cudanet_b200.h"

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

}  // namespace mayfly2
