"""PrefixCache over the sm_100a session with a bounded checkpoint pool: evicting checkpoints and
recycling their device buffers (B200StaticMG.state_into) must not change a single output bit
relative to keeping every checkpoint."""
import pytest
import torch

from fastworld_b200.config import SMALL
from fastworld_b200.prefix_cache import PrefixCache

pytestmark = pytest.mark.gpu


class LatentDecoder:
    """Decoder stand-in: the latent itself (as frames), so the served frames expose the latents."""

    def decode(self, lat):
        return lat[0, :3].float().clamp(-1, 1)

    def reset(self):
        pass

    def state(self):
        return None

    def load(self, st):
        pass


def test_bounded_pool_is_bitwise_equal_to_unbounded():
    from fastworld_b200.static import B200StaticMG
    from fastworld_b200.weights import synthetic_state_dict
    sd = synthetic_state_dict(SMALL, 0)
    trunk = [("img0", (k, c)) for k, c in zip("wwsadwsa", "uijklikl")]
    paths = [trunk, trunk[:5] + [("img0", ("q", "u"))] * 2, trunk[:3] + [("img0", ("d", "j"))],
             trunk[:7] + [("img0", ("s", "k"))], trunk[:5] + [("img0", ("a", "i"))] * 2]
    outs = []
    for bound in (None, 1):
        S = B200StaticMG(SMALL, sd)
        S.add_image("img0", seed=5, max_chunks=10)
        S.capture(warmup=1)
        cache = PrefixCache(S, LatentDecoder(), every=2, max_checkpoints=bound)
        got = []
        for p in paths:
            frames, _ = cache.serve(p)
            got.append(torch.stack(frames))
        torch.cuda.synchronize()
        assert S.device_status()[0] == 0
        outs.append((got, cache.n_evicted))
        S.graphs = {}
    assert outs[1][1] > 0                       # the bound was hit
    for a, b in zip(outs[0][0], outs[1][0]):
        assert torch.equal(a, b)
