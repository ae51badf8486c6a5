"""Status-synced host phases over gloo ranks (one rank raises, every rank stops at the same
point, collective counts stay equal) and the HBM pre-load check against a fake free size."""

import pytest
import torch

from difflet_b200.parallel.testing import run_ranks
from difflet_b200.utils import hbm


def _phase(rank, world):
    import torch.distributed as dist

    from difflet_b200.parallel.phase import RankFailureError, broadcast_object, collective_phase, rank0_call

    out = []
    try:
        with collective_phase("parse inputs"):
            if rank == 1:
                raise ValueError("bad request file")
    except RankFailureError as e:
        out.append(("peer", "rank 1" in str(e)))
    except ValueError:
        out.append(("own", True))
    # the next collective still pairs up on every rank
    t = torch.tensor([rank], dtype=torch.int64)
    dist.all_reduce(t)
    out.append(("sum", int(t)))
    v = rank0_call(lambda: {"steps": 28}, what="read config")
    out.append(("bcast", broadcast_object(v)["steps"]))
    with collective_phase("ok phase"):
        pass
    return out


@pytest.mark.multirank
def test_collective_phase_all_ranks_stop_together():
    res = run_ranks(_phase, 3, timeout=120)
    assert res[1][0] == ("own", True)
    assert res[0][0] == ("peer", True) and res[2][0] == ("peer", True)
    for r in res:
        assert r[1] == ("sum", 3) and r[2] == ("bcast", 28)


def test_hbm_check_fits_and_refuses():
    shapes = {"w": (1024, 1024)}
    w = hbm.weight_bytes(shapes, torch.bfloat16)
    assert w == 2 * 1024 * 1024
    hbm.check_fit(w, "cuda:0", what="tiny", free=10 * w)  # fits
    with pytest.raises(hbm.HbmBudgetError, match="needs"):
        hbm.check_fit(10 * w, "cuda:0", what="big", free=w)
    with pytest.raises(hbm.HbmBudgetError, match="weights fit"):
        hbm.check_fit(10 * w, "cuda:0", what="acts", free=2 * w, weights=w)
    hbm.check_fit(10**15, "cpu", what="cpu is not checked")
    # FLUX.1-dev in bf16 is about 23.8 GB of weights
    from difflet_b200.models.flux.config import get_config
    from difflet_b200.models.flux.model import FluxTransformer

    fw = hbm.weight_bytes(FluxTransformer.weight_shapes(get_config("flux-dev")), torch.bfloat16)
    assert 22e9 < fw < 25e9
