"""Expert parallelism at 4 and 8 GPUs (skipped with fewer): the decode layer
with 2 or 4 routed experts per rank, ragged batches and ranks without tokens,
every rank's output against the oracle.  Collected after the single- and
two-GPU tests."""
import pytest

from test_gpu_ep import _gpu_count, check_ranks, run_ranks
from test_gpu_moe import small_cfg


@pytest.mark.gpu
@pytest.mark.parametrize("world", [4, 8])
def test_ep_world_matches_oracle(cuda_lib, oracle, world):
    """The same decode layer at 4 and 8 ranks (2 or 4 routed experts per
    rank): ragged batches, ranks without tokens, then full batches."""
    if _gpu_count() < world:
        pytest.skip(f"needs {world} GPUs")
    cfg = small_cfg()
    H, O = cfg.hidden, oracle

    def toks(strm, T):
        return O.normal(strm, O.stream(0, 0, O.KIND_ACT), max(T, 1) * H, 1.0)[:T * H].reshape(T, H)

    batches = {r: [toks(600 + r, (3 * r + 1) % (cfg.max_tokens + 1)), toks(700 + r, 0 if r % 3 == 1 else 2),
                   toks(800 + r, cfg.max_tokens)] for r in range(world)}
    got = run_ranks(cuda_lib, cfg, 14, batches, world=world)
    check_ranks(O, cfg, 14, batches, got)
