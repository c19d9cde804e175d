#include <torch/extension.h>
void register_elementwise(pybind11::module& m) {}
