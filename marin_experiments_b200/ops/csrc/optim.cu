#include <torch/extension.h>
void register_optim(pybind11::module& m) {}
