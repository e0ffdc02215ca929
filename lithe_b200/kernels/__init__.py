"""sm_100a kernels behind LITHE's index-resident serving path (API of lithe/kernels).

* ``packed``  9-bit index packing (7 indices per uint64 word), the packed resident bank and
              the whole-adapter decode kernel.
* ``shared``  index-resident per-sample LoRA delta with the decode fused into the
              shrink / expand tiles (one launch per linear).
* ``layers``  nn.Module wrappers that route each sample of a batch to its own adapter.
"""
from ._launch import device_errors, raise_device_errors
from .layers import (IndexLoRALinear, PackedLoRALinear, PerSampleLoRALinear, SharedInputPrep, group_shared_inputs,
                     wrap_linears, wrap_packed)
from .packed import (PackedBank, PackedLayout, SlotLoader, decode_packed, flat_indices, pack_adapter,
                     pack_indices, split_decoded, unpack_indices)
from .shared import packed_codebook_lora_delta_, shared_codebook_lora_delta, shared_codebook_lora_delta_

__all__ = [
    "IndexLoRALinear", "PackedLoRALinear", "PerSampleLoRALinear", "SharedInputPrep", "group_shared_inputs",
    "wrap_linears", "wrap_packed",
    "PackedBank", "PackedLayout", "SlotLoader", "decode_packed", "flat_indices", "pack_adapter", "pack_indices",
    "split_decoded", "unpack_indices",
    "shared_codebook_lora_delta", "shared_codebook_lora_delta_", "packed_codebook_lora_delta_",
    "device_errors", "raise_device_errors",
]
