"""The drop-in boundary from a C host: tests/host_gguf.c reads one MoE layer
from a GGUF file with the reference's own gguf.c (under the tensor names of
infer.m:297-305), loads it with moe_load_layer and runs moe_forward.  The
GGUF file is written by gguf-py's GGUFWriter from oracle-generated experts;
the host's routing and outputs are checked against the oracle.  The program
is built by oracle/Makefile into oracle/_ref/host_gguf (from the reference
sources, where they are present).  Collected last."""
import os
import subprocess
import tempfile

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
HOST = os.path.join(os.path.dirname(HERE), "oracle", "_ref", "host_gguf")


def test_host_program_checks_its_arguments():
    if not os.path.exists(HOST):
        pytest.skip("oracle/_ref/host_gguf is not built (needs the reference's gguf.c)")
    r = subprocess.run([HOST], capture_output=True, text=True, timeout=60)
    assert r.returncode == 2 and "usage:" in r.stderr


@pytest.mark.gpu
def test_host_program_runs_a_gguf_layer(cuda_lib, oracle):
    gguf = pytest.importorskip("gguf")
    if not os.path.exists(HOST):
        pytest.skip("oracle/_ref/host_gguf is not built")
    from test_gpu_moe import GUARD, TOL, check_routing, oracle_cfg, rel_err, small_cfg
    O = oracle
    cfg = small_cfg()
    H, I, E, L, T, seed = cfg.hidden, cfg.intermediate, cfg.n_experts, 5, 5, 17
    gb, db = I * (H // 256) * 144, H * (I // 256) * 210
    blobs = {e: O.gen_expert(seed, L, e, H, I, O.TYPE_Q6_K) for e in range(E + 1)}  # [gate][up][down]
    router = O.normal(seed, O.stream(L, 0, O.KIND_ROUTER), E * H, 0.006).reshape(E, H)
    bias = O.normal(seed, O.stream(L, 0, O.KIND_BIAS), E, 0.01)
    tmp = tempfile.mkdtemp()
    path = os.path.join(tmp, "layer.gguf")
    q4, q6 = gguf.GGMLQuantizationType.Q4_K, gguf.GGMLQuantizationType.Q6_K

    def part(e, a, n, rows):
        return np.asarray(blobs[e], np.uint8).reshape(-1)[a:a + n].reshape(rows, -1)

    w = gguf.GGUFWriter(path, "deepseek2")
    w.add_tensor(f"blk.{L}.ffn_gate_exps.weight", np.stack([part(e, 0, gb, I) for e in range(E)]), raw_dtype=q4)
    w.add_tensor(f"blk.{L}.ffn_up_exps.weight", np.stack([part(e, gb, gb, I) for e in range(E)]), raw_dtype=q4)
    w.add_tensor(f"blk.{L}.ffn_down_exps.weight", np.stack([part(e, 2 * gb, db, H) for e in range(E)]), raw_dtype=q6)
    w.add_tensor(f"blk.{L}.ffn_gate_inp.weight", router.astype(np.float32))
    w.add_tensor(f"blk.{L}.exp_probs_b.bias", bias.astype(np.float32))
    w.add_tensor(f"blk.{L}.ffn_gate_shexp.weight", part(E, 0, gb, I), raw_dtype=q4)
    w.add_tensor(f"blk.{L}.ffn_up_shexp.weight", part(E, gb, gb, I), raw_dtype=q4)
    w.add_tensor(f"blk.{L}.ffn_down_shexp.weight", part(E, 2 * gb, db, H), raw_dtype=q6)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    h = O.normal(9, O.stream(L, 0, O.KIND_ACT), T * H, 1.0).reshape(T, H).astype(np.float32)
    h.tofile(os.path.join(tmp, "tokens.f32"))
    prefix = os.path.join(tmp, "res")
    args = [HOST, path, str(L), str(H), str(I), str(E), str(cfg.n_group), str(cfg.topk_group), str(cfg.top_k),
            os.path.join(tmp, "tokens.f32"), str(T), prefix]
    r = subprocess.run(args, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    out = np.fromfile(prefix + ".out", np.float32).reshape(T, H)
    idx = np.fromfile(prefix + ".idx", np.int32).reshape(T, cfg.top_k)
    wts = np.fromfile(prefix + ".w", np.float32).reshape(T, cfg.top_k)
    logits = (h.astype(np.float64) @ router.astype(np.float64).T).astype(np.float32)
    check_routing(O, cfg, logits, bias, idx, wts)
    ref, _, _, _ = O.moe_layer(oracle_cfg(cfg, O.TYPE_Q6_K), blobs, router, bias, h, force_idx=idx, force_w=wts)
    err = rel_err(out, ref)
    assert err < TOL and err < GUARD, err
