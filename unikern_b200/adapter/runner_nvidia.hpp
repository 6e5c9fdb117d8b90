// runner_nvidia.hpp -- the nvidia:cuda backend as the UNIKERN reference's own
// types see it: the translation unit a maintainer adds to the reference tree
// (beside src/runner.cpp, src/runner_ocl.cpp) to run the KML operator set on
// a B200 through libunikern_cuda.so.  Compiled against the reference's
// unmodified headers (include/unikern/{core,codegen,components}.hpp).
//
//   run_cuda ......... same shape as run_ocl / run_metal
//                      (include/unikern/codegen.hpp:104-117), returns the
//                      reference's RunOutcome (:49-83)
//   BackendNvidia .... an IBackend (include/unikern/components.hpp:14-33)
//   make_backends_with_nvidia
//                      make_backends (src/backends.cpp:82-90) with the nvidia
//                      backend appended, so the reference's fixed order of the
//                      first three is kept
//
// The reference's Vendor enum (components.hpp:11) has three values; the
// maintainer's patch appends Nvidia as the fourth (value 3, see
// kVendorNvidia), which this file uses without editing the header.
#pragma once

#include <memory>
#include <string>
#include <vector>

#include "unikern/codegen.hpp"
#include "unikern/components.hpp"
#include "unikern/core.hpp"

namespace unikern {

// the value Vendor::Nvidia takes once appended to the reference's enum
constexpr Vendor kVendorNvidia = static_cast<Vendor>(3);

// Run the declared tree on the current CUDA device: verify instance, e2e and
// kernel-only timing, the UNIKERN_RESULT line (in RunOutcome::log).  Nothing
// is generated or compiled, so workdir is not written.
RunOutcome run_cuda(const Solution& sol, const Hcs& hcs, const KmlTree& tree, const std::string& workdir);

class BackendNvidia : public IBackend {
 public:
  Vendor vendor() const override { return kVendorNvidia; }
  std::string name() const override { return "nvidia:cuda"; }
  // a CUDA device of compute capability 10.0 (B200) is visible
  bool available() const override;
  // provenance text: the kernels are precompiled for sm_100a
  std::string generate(const Solution& sol, const Hcs& hcs, const KmlTree& tree) const override;
  // GEMM operands larger than the device stream through a two-slot ring
  bool supports_streaming() const override { return true; }
  // the library's answer (uk_kml_describe's gap): fp32 and fp16 for all six
  // ops; int8, layouts other than NT and composite trees are refused with a
  // reason naming the field
  std::string capability_gap(const KmlTree& tree) const override;
};

std::vector<std::unique_ptr<IBackend>> make_backends_with_nvidia();

}  // namespace unikern
