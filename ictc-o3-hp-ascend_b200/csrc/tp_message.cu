// Instantiations of the graph-message kernels (destination-CSR forward, source-CSR adjoint).
#include "tp_kernels.cuh"

#include <vector>

namespace ictc {

template <int LI, int LE, int LO, int LAYOUT>
static void add_message(std::vector<Variant>& out) {
  // The forward keeps a node's whole output row in registers: one channel per lane,
  // or two when one warp covers a node (degrees up to 2, staged rows).
  out.push_back(make_variant<LI, LE, LO, 1, LAYOUT, kMessageForward>());
  if constexpr (LO <= 2) out.push_back(make_variant<LI, LE, LO, 2, LAYOUT, kMessageForward>());
  out.push_back(make_variant<LI, LE, LO, 1, LAYOUT, kMessageAdjoint>());
  out.push_back(make_variant<LI, LE, LO, 2, LAYOUT, kMessageAdjoint>());
}

template <int LI, int LE, int LO>
static void add_both(std::vector<Variant>& out) {
  add_message<LI, LE, LO, kIrMul>(out);
  add_message<LI, LE, LO, kMulIr>(out);
}

std::vector<Variant> message_variants() {
  std::vector<Variant> out;
  add_both<0, 1, 1>(out);
  add_both<1, 1, 1>(out);
  add_both<0, 2, 2>(out);
  add_both<2, 2, 2>(out);
  add_both<0, 3, 3>(out);
  add_both<3, 3, 3>(out);
  return out;
}

}  // namespace ictc
