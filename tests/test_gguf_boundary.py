"""CPU: the GGUF side of the drop-in boundary.  A GGUF file written by
gguf-py (GGUFWriter; the package the reference's gen_reference.py uses) holds
one layer's stacked expert tensors blk.L.ffn_{gate,up,down}_exps.weight in
ggml order (ne0 = columns, ne1 = rows, ne2 = experts; infer.m:1802-1823,
repack_experts.c:207-225).  The reference's own gguf.c reads them back, and
expert e is the byte slice [e * per-expert bytes, (e + 1) * per-expert
bytes) of each tensor: exactly what moe_load_layer takes (gate_exps +
e * gate bytes, ...).  The reference's quant.c dequantizes every slice to the
oracle's weights."""
import os
import tempfile

import numpy as np
import pytest

gguf = pytest.importorskip("gguf")

E, H, I, L = 4, 512, 256, 3


def test_gguf_expert_tensors_reach_the_loader_layout(oracle):
    O = oracle
    if not (O.ref_gguf_available() and O.ref_available()):
        pytest.skip("the reference's gguf.c / quant.c are not built (oracle/_ref)")
    q4, q6 = gguf.GGMLQuantizationType.Q4_K, gguf.GGMLQuantizationType.Q6_K
    mats = {
        "gate": ([O.gen_matrix(7, O.stream(L, e, O.KIND_GATE), O.TYPE_Q4_K, I, H, 0.02) for e in range(E)], q4, I, H),
        "up": ([O.gen_matrix(7, O.stream(L, e, O.KIND_UP), O.TYPE_Q4_K, I, H, 0.02) for e in range(E)], q4, I, H),
        "down": ([O.gen_matrix(7, O.stream(L, e, O.KIND_DOWN), O.TYPE_Q6_K, H, I, 0.02) for e in range(E)], q6, H, I),
    }
    path = os.path.join(tempfile.mkdtemp(), "layer.gguf")
    w = gguf.GGUFWriter(path, "deepseek2")
    for kind, (blobs, qt, rows, cols) in mats.items():
        stacked = np.stack([np.asarray(b, np.uint8).reshape(rows, -1) for b in blobs])  # [E][rows][row bytes]
        w.add_tensor(f"blk.{L}.ffn_{kind}_exps.weight", stacked, raw_dtype=qt)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    R = O.ref()
    for kind, (blobs, qt, rows, cols) in mats.items():
        got = O.ref_gguf_tensor(path, f"blk.{L}.ffn_{kind}_exps.weight")
        assert got is not None, kind
        dims, ty, data = got
        assert dims == [cols, rows, E], (kind, dims)
        assert ty == int(qt), (kind, ty)
        per = data.size // E
        assert per * E == data.size and per == np.asarray(blobs[0]).size
        for e in range(E):
            sl = np.ascontiguousarray(data[e * per:(e + 1) * per])
            assert np.array_equal(sl, np.asarray(blobs[e], np.uint8).reshape(-1)), (kind, e)
            ref = np.empty(rows * cols, np.float32)
            deq = R.dequantize_row_q6_K if qt == q6 else R.dequantize_row_q4_K
            deq(sl, ref, rows * cols)
            mine = O.dequant(np.asarray(blobs[e]), int(qt), rows * cols)
            assert np.array_equal(ref.view(np.uint32), np.asarray(mine, np.float32).view(np.uint32)), (kind, e)
    assert O.ref_gguf_tensor(path, f"blk.{L}.ffn_gate_exps.bias") is None
