#include <torch/extension.h>
void register_moe(pybind11::module& m) {}
