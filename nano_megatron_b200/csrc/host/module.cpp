// Host-only native runtime module (no CUDA dependency, importable on CPU hosts).
#include <torch/extension.h>

void register_data_loader(py::module& m);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "nano_megatron_b200 host runtime: data loading";
  register_data_loader(m);
}
