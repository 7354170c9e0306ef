// Name-only stand-in for the proxy library header, used solely to compile the
// reference's ops/partitioner.hpp into the oracle's reference shim. The
// partitioner header uses proxy only to declare a facade type at namespace
// scope; the shim calls the concrete partitioner classes directly, so these
// declarations never need a behaviour.
#pragma once
#define PRO_DEF_MEM_DISPATCH(name, func) struct name {}
namespace pro {
struct facade_builder {
  template <class Dispatch, class Signature> using add_convention = facade_builder;
  struct build {};
};
}  // namespace pro
