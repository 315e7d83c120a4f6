// Reader for PyTorch zip checkpoints (torch.save, zipfile format) holding f32 tensors: the model
// checkpoint kokoro-v1_0.pth (a dict of state dicts) and voice packs voices/*.pt (one tensor).
// Mirrors src/torchpt.rs: STORED zip entries only, a small pickle opcode set interpreted (never
// executed), and exactly the globals collections.OrderedDict, torch._utils._rebuild_tensor_v2 and
// torch.FloatStorage; anything else is refused with an error naming it.
#pragma once
#include <map>
#include <string>

#include "kk_weights.h"

namespace kk {

// {submodule: state_dict} -> "submodule.param" (a leading "module." inside a state dict is
// dropped, src/torchpt.rs:302-319); tensors contiguous row-major f32.
std::map<std::string, HostTensor> load_pth_checkpoint(const std::string& path);

// One tensor of shape [rows, 1, 256] (src/torchpt.rs:322-335).
HostTensor load_pth_voice(const std::string& path);

}  // namespace kk
