// TEST INFRASTRUCTURE ONLY.
//
// Link shim for the reference's runtime bench harness
// (bench/runtime/main.cpp, compiled unchanged from the reference sources by
// oracle/Makefile's `bench_runtime` target): the harness enumerates the CUDA
// slot through nert::CudaDevice() (main.cpp:192-203, include/nert/device.hpp:86);
// this definition hands it the B200 device handle instead, so the harness's
// own parity-and-timing cases (each op on the device against CpuDevice) run on
// nert::b200::Device(0) through the device seam. Its output labels the slot
// "CUDA".

#include "nert/device.hpp"

namespace nert {
namespace b200 {
const Device& Device(int ordinal);
} // namespace b200

const Device& CudaDevice() { return b200::Device(0); }

} // namespace nert
