// Hooks that moe_forward_grouped_gpu (ezzy0654/aps2026 src/tensor.cu:2790-2928)
// calls in place of its routing kernels and its un-permute, defined by
// tensor_ops_b2.cu over the aps2026_b200 C ABI.
//
// moe_forward_grouped_gpu also launches the reference's expert GEMMs, which
// are private to tensor.cu, so it cannot move out of that file. Instead the
// integration edits its body in two places (apply_moe_hook.py makes the edit
// mechanically): the scratch memsets + k_moe_top2 + k_moe_offsets_work +
// k_moe_fill_stable become one b2_dropin::moe_route call, and the
// k_moe_combine launch becomes one b2_dropin::moe_combine call. The outputs
// are written into the reference's own MoeScratch buffers in the formats its
// grouped GEMMs read (u8 routes, expert-ordered assignment rows, 64- and
// 128-row work queues with 0xFFFFFFFF for unused entries), bit for bit what
// the replaced kernels wrote.
#pragma once

#include <cstddef>
#include <cstdint>

namespace b2_dropin {

// Top-2 routing of router_logits [rows, NUM_EXPERTS] on the legacy stream:
// routes [rows, 2], counts [E], offsets [E + 1], assignment_rows and
// route_positions [2 rows], and the two work queues of lengths
// ceil(2 rows / 64) + E and ceil(2 rows / 128) + E. Throws
// std::invalid_argument / std::runtime_error like the reference.
void moe_route(const float* router_logits, std::size_t rows, std::uint8_t* routes,
               std::uint32_t* counts, std::uint32_t* offsets, std::uint32_t* assignment_rows,
               std::uint32_t* route_positions, std::uint32_t* work_expert64,
               std::uint32_t* work_start64, std::uint32_t* work_expert128,
               std::uint32_t* work_start128);

// out[t, :] = 0.5 * expert_out[p_lo, :] + 0.5 * expert_out[p_hi, :] for
// t < rows, expert_out being [expert_rows, h] in expert order.
void moe_combine(const float* expert_out, std::size_t expert_rows, const std::uint8_t* routes,
                 const std::uint32_t* route_positions, float* out, std::size_t rows,
                 std::size_t h);

}  // namespace b2_dropin
