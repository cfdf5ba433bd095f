// TEST INFRASTRUCTURE ONLY (oracle). Stand-in for the reference's
// include/soar/nn/module.hpp: just the parameters() list that the reference's
// header-only soar::utils::ModelEMA (include/soar/utils/ema.hpp) reads, so that
// header compiles unmodified in oracle/ref_shim.cpp.
#pragma once

#include <memory>
#include <vector>

#include <soar/tensor/tensor.hpp>

namespace soar::nn {

class Module {
public:
    explicit Module(std::vector<TensorPtr> params) : params_(std::move(params)) {}
    [[nodiscard]] std::vector<TensorPtr> parameters() const { return params_; }

private:
    std::vector<TensorPtr> params_;
};

}  // namespace soar::nn
