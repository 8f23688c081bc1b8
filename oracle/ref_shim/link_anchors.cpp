// Out-of-line definitions of mlx::core::Primitive's non-pure virtuals.  The
// shim only calls free template functions; these anchor the class's vtable
// and type information so the shared object links without the rest of MLX.
// They are never executed.
#include "mlx/primitives.h"

#include <stdexcept>

namespace mlx::core {
std::vector<array> Primitive::jvp(const std::vector<array>&, const std::vector<array>&,
                                  const std::vector<int>&) {
  throw std::logic_error("not part of the shim");
}
std::vector<array> Primitive::vjp(const std::vector<array>&, const std::vector<array>&,
                                  const std::vector<int>&, const std::vector<array>&) {
  throw std::logic_error("not part of the shim");
}
std::pair<std::vector<array>, std::vector<int>> Primitive::vmap(const std::vector<array>&,
                                                                const std::vector<int>&) {
  throw std::logic_error("not part of the shim");
}
std::vector<Shape> Primitive::output_shapes(const std::vector<array>&) {
  throw std::logic_error("not part of the shim");
}
}  // namespace mlx::core
