"""CPU: the packed-weight layout (section offsets and sizes, alignment), argument checks of the
packing entry points, and the file format's round trip."""
import pytest
import torch

from muxi_race_b200 import _lib
from muxi_race_b200.packed import KINDS, PackedWeights, packed_layout


@pytest.mark.parametrize("kind", sorted(KINDS))
@pytest.mark.parametrize("E,H,I", [(8, 1024, 512), (256, 7168, 2048), (6, 136, 208)])
def test_layout(kind, E, H, I):
    off, total = packed_layout(E, H, I, kind)
    q = kind in ("int8", "fp8")
    elt = 1 if q else 2
    sizes = [E * 2 * I * H * elt, E * 2 * I * 4 if q else 0, E * H * I * elt, E * H * 4 if q else 0]
    assert off[0] == 0 and all(o % 256 == 0 for o in off) and total % 256 == 0
    for i in range(3):
        assert off[i + 1] >= off[i] + sizes[i] and off[i + 1] - (off[i] + sizes[i]) < 256
    assert total >= off[3] + sizes[3] and total - (off[3] + sizes[3]) < 256
    if not q:
        assert off[1] == off[2] and off[3] == total


def test_bad_arguments():
    lib = _lib.lib()
    with pytest.raises(_lib.MoeError, match="kind"):
        _lib.call("moe_packed_weights_layout", 8, 1024, 512, _lib.MOE_F32, None, None)
    rc = lib.moe_pack_weights(None, None, None, _lib.MOE_F16, 8, 1024, 512, _lib.MOE_BF16, None, 0, None)
    assert rc == -1 and b"dtype" in lib.moe_last_error()
    rc = lib.moe_pack_weights(None, None, None, _lib.MOE_F16, 8, 1000, 512, _lib.MOE_I8, None, 0, None)
    assert rc == -1 and b"multiples of 16" in lib.moe_last_error()
    rc = lib.moe_fused_packed(None, None, _lib.MOE_F32, None, _lib.MOE_I32, None, _lib.MOE_F32, None, 4, 1024, 512,
                              8, 2, _lib.MOE_F16, None, 0, None)
    assert rc == -1 and b"kind" in lib.moe_last_error()
    # workspace sizes follow the route of the kind
    assert lib.moe_fused_packed_workspace_bytes(64, 2, 8, 1024, 512, _lib.MOE_I8, _lib.MOE_F16) == \
        lib.moe_fused_int8_workspace_bytes(64, 2, 8, 1024, 512, _lib.MOE_F16)
    assert lib.moe_fused_packed_workspace_bytes(64, 2, 8, 1024, 512, _lib.MOE_F16, _lib.MOE_F16) == \
        lib.moe_fused_workspace_bytes(64, 2, 8, 1024, 512, _lib.MOE_F16)


def test_file_round_trip(tmp_path):
    E, H, I = 4, 256, 128
    _, total = packed_layout(E, H, I, "int8")
    g = torch.Generator().manual_seed(0)
    blob = torch.randint(0, 256, (total,), generator=g, dtype=torch.uint8)
    p = PackedWeights(blob, E, H, I, "int8")
    path = tmp_path / "w.bin"
    p.save(str(path))
    back = PackedWeights.load(str(path), device="cpu")
    assert (back.E, back.H, back.I, back.kind) == (E, H, I, "int8")
    assert torch.equal(back.blob, blob)
    # a file whose size does not match its header's layout is refused
    raw = path.read_bytes()
    (tmp_path / "short.bin").write_bytes(raw[:-256])
    with pytest.raises(ValueError, match="layout needs"):
        PackedWeights.load(str(tmp_path / "short.bin"), device="cpu")
