// Shared host-side declarations for the extension.
#pragma once

#include <cuda.h>
#include <pybind11/pybind11.h>
#include <torch/extension.h>

namespace py = pybind11;

namespace dst {

// Per-device int32 status word that bounded device-side waits write their
// error code into (0 = ok). Allocated lazily, once per device.
int* status_ptr();

int num_sms();

CUtensorMap make_tmap_bf16(const void* base, uint64_t inner, uint64_t outer, uint64_t ld, uint32_t box_inner,
                           uint32_t box_outer);

}  // namespace dst

void register_gemm(pybind11::module& m);
void register_norm(pybind11::module& m);
void register_embed(pybind11::module& m);
void register_adam(pybind11::module& m);
void register_ce(pybind11::module& m);
void register_attn_tc(pybind11::module& m);
void register_symm(pybind11::module& m);
void register_tp(pybind11::module& m);
