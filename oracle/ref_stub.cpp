// TEST INFRASTRUCTURE ONLY -- part of the parity oracle, never shipped.
//
// Host-side stand-ins for the reference's XRT device layer, so that the
// reference's own host-CPU encoders (runtime/src/encoders/bert_encoder.cpp and
// runtime/src/vit/encoder.cpp, compiled from the reference tree where they
// lie) link without XRT.
//
// The oracle runs the reference with `--npu-ops` empty, which is its default
// (runtime/include/common/npu_ops_flag.hpp:96-103): every GEMM goes to
// hostconv::gemm_nt, every LayerNorm/softmax/GELU to the *_cpu passes.  None of
// the array methods below is reachable on that path, so each one throws by
// name: reaching one means the oracle is not running the host path and its
// answer must not be trusted.  The one exception is the array emulation
// below, which a driver switches on explicitly for an int8 container.
//
// Symbols provided (the set the linker reports missing when the sources in
// oracle/Makefile's REF_SRCS are linked alone):
//   npu::Device::{Device,~Device}                    runtime/include/runtime/device.hpp:29-38
//   npu::Design::{Design,~Design,stage,bind,...}     runtime/include/runtime/design.hpp:199-263
// (npue::gemma_rope_tables, which the rotary host path of
// nomic_bert_rope_swiglu calls, comes from the reference's own
// encoders/gemma_kernels.cpp, linked alongside.)
// (npue::whisper::NpuAttention::run comes from the reference's own
// whisper/attention_npu.cpp, linked for the ViT path; it is not reached.)

#include <cstdint>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

#include "ref_array.hpp"
#include "runtime/design.hpp"
#include "runtime/device.hpp"
#include "runtime/model.hpp"

namespace {
[[noreturn]] void unreachable(const char *what) {
  throw std::runtime_error(std::string("oracle host stub: ") + what +
                           " reached -- the oracle must run the reference's "
                           "host-CPU path only (--npu-ops empty)");
}
}  // namespace

namespace npu {

struct Device::Impl {};
Device::Device() {}
Device::~Device() {}

}  // namespace npu

// What the stand-in design reports for a pre-tiled container (gemm_layout
// "pretiled_bf16"), set by the drivers before an encoder is built: the
// operands' layout_hash, so that stage_all's design/model layout check
// (bert_encoder.cpp:41-150) passes as it does with a matching design set,
// and the operand width, 1 for an int8 container, which is what makes
// stage_all load .wscale / .asmooth and the host GEMM divide A by .asmooth.
std::string nebw_oracle_b_layout_hash;
size_t nebw_oracle_a_elem_bytes = 2;

// The stand-in design matches the container, as a design set exported for it
// would: the operands' layout hash, and int8 operands for a_dtype "i8".
// Called by the drivers before they build an encoder.
void nebw_oracle_describe_design(const npue::File &f) {
  std::string layout, a_dtype;
  try {
    layout = f.config_string("gemm_layout");
  } catch (const std::exception &) {
  }
  try {
    a_dtype = f.config_string("a_dtype");
  } catch (const std::exception &) {
  }
  nebw_oracle_b_layout_hash.clear();
  nebw_oracle_a_elem_bytes = 2;
  if (layout == "host") return;
  nebw_oracle_b_layout_hash = f.info("layer.0.qkv").layout_hash;
  if (a_dtype == "i8" || a_dtype == "I8") nebw_oracle_a_elem_bytes = 1;  // BERT / ViT packers
}

// ---- array emulation: an int8 container with its GEMMs on the array ------
// With nebw_array_on set (by a driver, around one encode), the stand-in
// design does what an int8 GEMM design does in BertEncoder::gemm's array
// branch (bert_encoder.cpp:763-810): the host quantises A into the design's
// A slot, the dispatch multiplies it by the staged int8 operand into int32
// C, and the host dequantises C from the C slot.  The product is the
// array's: a sum of int8 x int8 products in int32 is exact, so any order
// gives its bits.  The driver registers, by the panel address stage_all()
// hands to stage() (the container mapping, npue::gemm_b_panel), each
// operand's int8 [K, N], and sizes the A and C slots for the pass.
std::map<const void *, NebwArrayOperand> nebw_array_registry;
bool nebw_array_on = false;
int64_t nebw_array_rows = 0;
std::vector<int8_t> nebw_array_a;    // the A slot
std::vector<int32_t> nebw_array_c;   // the C slot

namespace {
std::map<size_t, const NebwArrayOperand *> g_slot_operand;
size_t g_bound[3] = {0, 0, 0};
}  // namespace

namespace npu {

struct Design::Impl {};
Design::Design(Device &dev, const std::string &dir) : dev_(&dev) {
  info_.name = dir;  // used only as a cache-key label by host_b.hpp
  info_.b_layout_hash = nebw_oracle_b_layout_hash;
  info_.a_elem_bytes = nebw_oracle_a_elem_bytes;
  // NpuGemm::alloc_buffers (runtime/src/whisper/npu_ops.cpp:29-32) reads the
  // A and C entries of buffer_bytes; a host-layout run never uses the sizes.
  info_.buffer_bytes.assign(3, 0);
}
Design::~Design() {}

void Design::run(const std::vector<const void *> &, void *) { unreachable("Design::run"); }
void Design::dispatch_only() {
  if (!nebw_array_on) unreachable("Design::dispatch_only");
  const auto it = g_slot_operand.find(g_bound[1]);
  if (it == g_slot_operand.end()) unreachable("dispatch of an operand that was never staged");
  const NebwArrayOperand &w = *it->second;
  const int64_t M = nebw_array_rows, K = w.K, N = w.N;
  if (static_cast<int64_t>(nebw_array_a.size()) < M * K + 64 ||
      static_cast<int64_t>(nebw_array_c.size()) < M * N + 16)
    unreachable("dispatch larger than the A / C slots");
  const int8_t *A = nebw_array_slot(nebw_array_a);
  int32_t *Cs = nebw_array_slot(nebw_array_c);
  std::vector<int32_t> acc(static_cast<size_t>(N));
  for (int64_t r = 0; r < M; ++r) {
    std::fill(acc.begin(), acc.end(), 0);
    const int8_t *a = A + r * K;
    for (int64_t k = 0; k < K; ++k) {
      const int32_t av = a[k];
      const int8_t *wr = w.kn.data() + k * N;
      for (int64_t n = 0; n < N; ++n) acc[n] += av * wr[n];
    }
    std::copy(acc.begin(), acc.end(), Cs + r * N);
  }
}
void Design::bind_instr(size_t) { unreachable("Design::bind_instr"); }
// Staging a pre-tiled weight panel uploads nothing here: the host GEMM reads
// the operand from the container (host_b.hpp) by the slot it was recorded
// under, so a fresh slot number per call is all stage_all needs.  A host-
// layout container never stages.
size_t Design::stage(size_t, const void *data, size_t) {
  static size_t staged = size_t{1} << 32;  // apart from host_layout's slot numbers
  ++staged;
  if (nebw_array_on) {
    const auto it = nebw_array_registry.find(data);
    if (it != nebw_array_registry.end()) g_slot_operand[staged] = &it->second;
  }
  return staged;
}
// VitEncoder::stage_all -> NpuGemm::alloc_buffers (runtime/src/whisper/
// npu_ops.cpp:29-32) reserves the design's A and C slots even on a
// host-layout container, whose GEMMs never touch them; the slot numbers are
// returned and never used.
size_t Design::stage_alloc(size_t arg, size_t) { return arg; }
// Off the array emulation, the one method that does not throw:
// BertEncoder::run() takes the FFN-down A-slot address unconditionally when
// it builds its FusedNext/FusedNextBf16 descriptors (bert_encoder.cpp:
// 1529-1541) and only writes through it when the GEMMs are on the array.  On
// the host path the address is built and never used, so a null answer is
// exact; a write through it would fault loudly rather than corrupt anything.
// Under the emulation, the A and C slots.
void *Design::slot_ptr(size_t arg, size_t) {
  if (!nebw_array_on) return nullptr;
  if (arg == 0) return nebw_array_slot(nebw_array_a);
  if (arg == 2) return nebw_array_slot(nebw_array_c);
  unreachable("Design::slot_ptr of a weight argument");
}
void Design::bind(size_t arg, size_t slot) {
  if (!nebw_array_on || arg > 2) unreachable("Design::bind");
  g_bound[arg] = slot;
}
void *Design::host_ptr(size_t) { unreachable("Design::host_ptr"); }
void Design::sync_to_device(size_t, size_t) { unreachable("Design::sync_to_device"); }
void Design::sync_from_device(size_t, size_t) { unreachable("Design::sync_from_device"); }
// The slots are host memory here: nothing to copy.
void Design::sync_slot_to_device(size_t, size_t, size_t) {
  if (!nebw_array_on) unreachable("Design::sync_slot_to_device");
}
void Design::sync_slot_from_device(size_t, size_t, size_t) {
  if (!nebw_array_on) unreachable("Design::sync_slot_from_device");
}

}  // namespace npu


