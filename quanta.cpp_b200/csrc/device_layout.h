// The device's row order for the fused matrices, on the host, and a .qnt writer that stores them pre-packed.
//
// The engine fuses each layer's q, k and v into one matrix whose rows are pair-interleaved per head (row i and
// i + head_dim / 2 of a head adjacent, so one thread applies bias and RoPE to a rotation pair), and gate and up into
// one matrix interleaved per 32 rows (the SwiGLU pair in one CTA).  export_device_layout writes a copy of a .qnt file
// with those matrices (and the q|k|v bias in the same order) added as ordinary tensors:
//   b200.layout                       f32 [1]  the layout version (1)
//   b200.layers.<l>.qkv               the fused q|k|v, the dtype of q/k/v
//   b200.layers.<l>.qkv_bias          f32 [rows] (files with q|k|v biases)
//   b200.layers.<l>.gate_up           the fused gate|up, the dtype of gate/up
// Every original tensor is kept, byte for byte, so the reference's reader loads the file unchanged (it ignores
// tensors it does not look up), and the engine uploads the fused tensors as they are, without reordering rows.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "qnt_file.h"

namespace qb {

constexpr int kDeviceLayoutVersion = 1;

struct FusedHost {
    int dtype = 0, rows = 0, cols = 0;
    std::vector<uint8_t> q;   // quants, row-major
    std::vector<uint16_t> d;  // fp16 block scales, [rows][cols / 32]
};

// mode 0: q|k|v pair-interleaved per head of head_dim; mode 1: gate|up interleaved per 32 rows.  Throws on mismatched
// dtypes or widths.
FusedHost fuse_rows(const std::vector<const HostTensor*>& parts, int mode, int head_dim);
// The q, k and v biases (f32) in fuse_rows' mode-0 row order.
std::vector<float> fuse_qkv_bias(const std::vector<const HostTensor*>& biases, int head_dim);
// True when `packed` has the fused matrix's dtype and shape and, on a sample of rows spread over it (the first and last
// included), the parts' rows in fuse_rows' order: a stale or foreign pre-packed tensor is not uploaded.
bool packed_rows_match(const HostTensor& packed, const std::vector<const HostTensor*>& parts, int mode, int head_dim);

// Writes in_path's tensors plus the pre-packed ones to out_path.  Returns false with *err on failure.
bool export_device_layout(const std::string& in_path, const std::string& out_path, std::string* err);

}  // namespace qb
