"""The C-ABI weight packer (glad_pack_layout / glad_pack_weights / glad_unpack_weights)
builds the same broadcast blob as the Python PackedWeights, and unpacks it exactly."""
import pytest
import torch

from rl_quant_b200 import _native as N
from rl_quant_b200.glad_model import build_glad
from rl_quant_b200.weight_sync import PackedWeights

pytestmark = pytest.mark.gpu


def test_c_abi_pack_equals_packed_weights():
    lib = N.load()
    m = build_glad(seed=0, critic_seed=2).half().cuda()
    tensors = []
    seen = set()
    for mod in m.modules():
        for t in list(mod.parameters(recurse=False)) + [b for n, b in mod.named_buffers(recurse=False)
                                                       if not n.startswith("_") and n != "num_batches_tracked"]:
            if t.data_ptr() not in seen:
                seen.add(t.data_ptr())
                tensors.append(t.detach().clone())
    packed = PackedWeights(m)
    items = (N.GladPackItem * len(tensors))(*[N.GladPackItem(t.data_ptr(), t.numel() * t.element_size(), 0)
                                              for t in tensors])
    total = lib.glad_pack_layout(items, len(tensors))
    assert total == packed.blob.numel()
    blob = torch.zeros(total, dtype=torch.uint8, device="cuda")
    N.check(lib.glad_pack_weights(items, len(tensors), blob.data_ptr(), total, N.stream_handle()), "pack")
    torch.cuda.synchronize()
    assert torch.equal(blob, packed.blob)
    outs = [torch.zeros_like(t) for t in tensors]
    for it, o in zip(items, outs):
        it.tensor = o.data_ptr()
    N.check(lib.glad_unpack_weights(items, len(tensors), blob.data_ptr(), total, N.stream_handle()), "unpack")
    torch.cuda.synchronize()
    assert all(torch.equal(a, b) for a, b in zip(outs, tensors))
