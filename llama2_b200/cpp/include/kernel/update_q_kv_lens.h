// launch_update_q_kv_lens — the reference's include/kernel/update_q_kv_lens.h:6-9 signature.
#pragma once

template <typename T>
class Tensor;

// kv_lens += q_lens; max_q_len / max_kv_len (1 element each) receive the
// maxima. As in the reference, host tensors receive them synchronously
// (pinned-host afterwards); device tensors keep them on the device.
void launch_update_q_kv_lens(const Tensor<unsigned int> &q_lens, // (batch)
                             Tensor<unsigned int> &kv_lens,      // (batch)
                             Tensor<unsigned int> &max_q_len,    // (1)
                             Tensor<unsigned int> &max_kv_len);  // (1)
