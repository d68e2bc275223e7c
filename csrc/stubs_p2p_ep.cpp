// Placeholder registrations replaced as the P2P and EP layers land.
#include <pybind11/pybind11.h>
namespace py = pybind11;
void register_p2p(py::module_& m) { m.def_submodule("p2p", "kiwi::p2p (NVLink peer memory)"); }
void register_ep(py::module_& m) { m.def_submodule("ep", "kiwi::ep (expert-parallel MoE)"); }
