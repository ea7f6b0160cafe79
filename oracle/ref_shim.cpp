// ref_shim.cpp -- exposes the reference's own C++ assignment solver
// (src/cpu/matching.cpp:71-571 of AndyBarcia/mask_loss) through a C ABI so
// the tests and the CPU baseline can call it on fp64 cost slices.
//
// TEST INFRASTRUCTURE ONLY.  The reference source is #included from where it
// lies (REF_SRC/cpu/matching.cpp, passed by oracle/Makefile); nothing from it
// is copied into this repository.  The two CUDA-side functions that
// matching.cpp declares but this shim never reaches are defined as stubs that
// raise, so the translation unit links without the reference's CUDA code.
#include "matching.cpp"

#include <thread>

torch::Tensor pairwise_mask_loss_forward(
    const torch::Tensor&, const torch::Tensor&, const torch::Tensor&, const torch::Tensor&,
    const float, const float, const float, const float, int64_t, const float, const float,
    const float, const float, const float, const float, bool, bool) {
    TORCH_CHECK(false, "ref_shim: pairwise_mask_loss_forward is not available");
}

std::vector<torch::Tensor> mask_matching_forward(
    const torch::Tensor&, const torch::Tensor&, const torch::Tensor&, const torch::Tensor&,
    const float, const float, const float, const float, const float, const float,
    const float, const float, const int64_t, const int64_t, const double, const bool,
    const bool, const int64_t, const bool, const bool) {
    TORCH_CHECK(false, "ref_shim: mask_matching_forward is not available");
}

extern "C" int ref_assign_slice(const double* cost, int64_t Q, int64_t GT_out, double thr,
                                int64_t topk, int strategy, int64_t* p2g, int64_t* prnd) {
    try {
        assign_predictions_for_slice(cost, Q, GT_out, thr, topk,
                                     static_cast<MatchingStrategy>(strategy),
                                     reinterpret_cast<long*>(p2g), reinterpret_cast<long*>(prnd));
        return 0;
    } catch (...) {
        return 2;
    }
}

// All slices of an (N,Q,GT_out) batch on `threads` host threads, chunked the
// way at::parallel_for splits the L*B range in src/cpu/matching.cpp:690.
extern "C" int ref_assign_batch(const double* cost, int64_t N, int64_t Q, int64_t GT_out,
                                double thr, int64_t topk, int strategy, int64_t* p2g,
                                int64_t* prnd, int threads) {
    if (threads < 1) threads = 1;
    std::vector<std::thread> pool;
    std::vector<int> rcs(threads, 0);
    const int64_t chunk = (N + threads - 1) / threads;
    for (int t = 0; t < threads; ++t) {
        pool.emplace_back([&, t]() {
            for (int64_t i = t * chunk; i < std::min<int64_t>(N, (t + 1) * chunk); ++i) {
                int rc = ref_assign_slice(cost + i * Q * GT_out, Q, GT_out, thr, topk, strategy,
                                          p2g + i * Q, prnd + i * Q);
                if (rc) rcs[t] = rc;
            }
        });
    }
    for (auto& th : pool) th.join();
    for (int rc : rcs) if (rc) return rc;
    return 0;
}
