#include <torch/extension.h>
void register_attention(pybind11::module& m) {}
