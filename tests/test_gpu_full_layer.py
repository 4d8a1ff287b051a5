"""GPU parity at the benchmark's full size: one Qwen3-14B-shaped decoder
layer (q/k/v/o/gate/up/down, 330.3 M BF16 weights) decoded by ONE batched
launch (aib_decode_bf16_batch, 7 tensors, ~2.9 waves of CTAs), in the three
chunkings the benchmark and the tensor-parallel stores use, with the
stream in the reference layout and in the striped device layout:
  * the reference's default, 1024 symbols for every tensor;
  * TP-ready (whole chunks per rank up to TP 8): o_proj 640, down_proj 1088;
  * the TP-8 store: 256, with o_proj 320 and down_proj 128.
Every output must equal the source weights bit for bit and the CPU oracle's
reconstruction (reference compressed_store.py:186-240 with the numba CPU
decoder, cpu_decode.py:67-113)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

LAYER = [("q_proj", 5120, 5120), ("k_proj", 1024, 5120), ("v_proj", 1024, 5120),
         ("o_proj", 5120, 5120), ("gate_proj", 17408, 5120), ("up_proj", 17408, 5120),
         ("down_proj", 5120, 17408)]
CHUNKINGS = {
    "default-1024": {},
    "tp-ready-640-1088": {"o_proj": 640, "down_proj": 1088},
    "tp8-256": {"*": 256, "o_proj": 320, "down_proj": 128},
}


@pytest.fixture(scope="module")
def weights():
    g = torch.Generator().manual_seed(2024)
    return [(name, (torch.randn(r, c, generator=g) * 0.02).to(torch.bfloat16)) for name, r, c in LAYER]


@pytest.mark.parametrize("layout", ["reference", "striped"])
@pytest.mark.parametrize("chunking", sorted(CHUNKINGS))
def test_full_14b_layer_one_launch_is_bit_exact(weights, chunking, layout):
    from afterimage_b200.runtime import _device
    from afterimage_b200.runtime.compressed_store import compress_layer
    from afterimage_b200.runtime.layer_decode import LayerDecoder, upload_layer
    dev = torch.device("cuda", 0)
    sizes = CHUNKINGS[chunking]
    layers = [compress_layer(W, chunk_size=sizes.get(name, sizes.get("*", 1024))) for name, W in weights]
    resident = [upload_layer(layer, dev, striped=layout == "striped") for layer in layers]
    outs = [torch.full(W.shape, float("nan"), dtype=torch.bfloat16, device=dev) for _, W in weights]
    dec = LayerDecoder(dev)
    descs = dec.descriptors(resident, outs)
    dec.launch(descs, len(resident))
    assert dec.launches == 1
    torch.cuda.synchronize(dev)
    _device.check_status(dev)
    for (name, W), layer, out in zip(weights, layers, outs):
        got = out.cpu().view(torch.int16).reshape(-1)
        assert torch.equal(got, W.view(torch.int16).reshape(-1)), (chunking, name)
        ref = O.decompress(layer.encoded, layer.sign_mantissa.numpy()).view(np.int16)
        assert np.array_equal(got.numpy(), ref), (chunking, name)
    # a second launch over the same descriptors (the benchmark's repeated step) is unchanged
    for o in outs:
        o.fill_(float("nan"))
    dec.launch(descs, len(resident))
    torch.cuda.synchronize(dev)
    _device.check_status(dev)
    for (name, W), out in zip(weights, outs):
        assert torch.equal(out.cpu().view(torch.int16), W.view(torch.int16)), (chunking, name, "repeat")
