// TEST INFRASTRUCTURE ONLY -- part of the parity oracle, never shipped.
//
// The array emulation of the stand-in design (oracle/ref_stub.cpp), shared
// with the driver that switches it on (oracle/ref_driver.cpp,
// nebw_ref_encode_array).  Under it an int8 GEMM design's dispatch is the
// exact int32 product of the A slot's int8 rows and the staged operand.
#pragma once

#include <cstdint>
#include <map>
#include <vector>

struct NebwArrayOperand {
  std::vector<int8_t> kn;  // the operand as int8 [K, N], row-major
  int64_t K = 0, N = 0;
};

// operands by the panel address stage_all() hands to Design::stage
extern std::map<const void *, NebwArrayOperand> nebw_array_registry;
extern bool nebw_array_on;          // the emulation is active
extern int64_t nebw_array_rows;     // rows of every dispatch (BertEncoder::rows)
// the A and C slots' storage: rows x max K int8 and rows x max N int32, each
// with 64 bytes to spare so that the slot itself starts 64-byte aligned (the
// reference's streaming loads want 32)
extern std::vector<int8_t> nebw_array_a;
extern std::vector<int32_t> nebw_array_c;

template <typename T>
T *nebw_array_slot(std::vector<T> &v) {
  const uintptr_t p = reinterpret_cast<uintptr_t>(v.data());
  return reinterpret_cast<T *>((p + 63) & ~uintptr_t{63});
}
