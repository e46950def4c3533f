"""CPU checks of the tcgen05 attention kernels' barrier protocols (models in
kernel_protocols.py): under random interleavings of all roles, random TMA
latencies and an in-order tensor pipe, no role deadlocks, no wait sees its
barrier two phases ahead (a parity hang on the GPU), and no buffer or TMEM
range is overwritten before its consumer read it -- for every tile count up to
6, with and without the pair bias.  Planted mistakes (one wait removed, on the
CPU) are caught, so the models can fail."""
import pytest

import kernel_protocols as kp


@pytest.mark.parametrize("pair", [False, True])
def test_forward_protocol(pair):
    for n_kt in range(0, 7):
        for seed in range(60):
            kp.forward(n_kt, pair, seed)


@pytest.mark.parametrize("pair", [False, True])
@pytest.mark.parametrize("slow_tma", [False, True])
def test_backward_protocol(pair, slow_tma):
    for tiles in range(1, 7):
        for seed in range(40):
            kp.backward(tiles, pair, seed, slow_tma=slow_tma)


def _caught(fn, plant, **kw):
    for seed in range(200):
        try:
            fn(seed=seed, plant=plant, **kw)
        except kp.ProtocolBug:
            return True
    return False


@pytest.mark.parametrize("plant", ["KVEmpty0", "KVEmpty1", "PairEmpty0", "PFull0", "SFull1", "KFull1", "OStep",
                                   "OFinal", "PairFull1"])
def test_forward_planted_mistake_is_caught(plant):
    assert _caught(kp.forward, plant, n_kt=5, pair=True)


@pytest.mark.parametrize("plant", ["QEmpty0", "DSEmpty0", "DQEmpty", "bulk_wait_read0", "TileEmpty0",
                                   "SFull1", "PFull1", "QFull1", "DQFull", "TileFull0", "PairFull1", "KVTmem",
                                   "PairFull3"])
def test_backward_planted_mistake_is_caught(plant):
    kw = dict(T=5, pair=True)
    assert (_caught(kp.backward, plant, **kw)
            or _caught(kp.backward, plant, slow_roles=("provider",), **kw)
            or _caught(kp.backward, plant, slow_roles=("dq0", "dq1", "dq2", "dq3"), **kw)
            or _caught(kp.backward, plant, slow_tma=True, **kw)
            or _caught(kp.backward, plant, slow_roles=("ew0", "ew1"), **kw))


@pytest.mark.parametrize("plant", ["PairEmpty0", "PairEmpty3"])
def test_backward_pair_empty_is_implied(plant):
    """With the pair halves of tile t issued by the Q/dO producer after its
    QEmpty(t-2) wait, the products of tile t-2 -- and so the elementwise reads
    of pair halves 2t-4 and 2t-3, the previous contents of the two slots --
    are already done: the PairEmpty waits never wait (the model finds no
    hazard without them).  The kernel keeps them as a guard."""
    for kw in (dict(), dict(slow_tma=True), dict(slow_roles=("ew0", "ew1"))):
        assert not _caught(kp.backward, plant, T=5, pair=True, **kw)


def test_backward_per_half_store_wait_is_implied():
    """The MMA warp's bulk_wait_read<2> after each dS store is implied by the
    bulk_wait_read<0> before every dQ commit (the model finds no hazard without
    it): the store two halves back is always already read."""
    assert not _caught(kp.backward, "bulk_wait_read2", T=5, pair=True)


@pytest.mark.parametrize("slow_tma", [False, True])
def test_backward128_protocol(slow_tma):
    for steps in range(0, 9):
        for seed in range(40):
            kp.backward128(steps, seed, slow_tma=slow_tma)


@pytest.mark.parametrize("plant", ["QEmpty0", "QEmpty2", "QFull1", "QFull2", "PFull0", "PFull1", "SFull1",
                                   "DQEmpty0", "DQEmpty1", "DQFull1", "DSEmpty0", "DSEmpty1", "TileFull0",
                                   "TileEmpty1"])
def test_backward128_planted_mistake_is_caught(plant):
    assert _caught(kp.backward128, plant, T=7) or _caught(kp.backward128, plant, T=7, slow_tma=True)


@pytest.mark.parametrize("stages,pair", [(2, False), (3, False), (2, True)])
@pytest.mark.parametrize("slow_tma", [False, True])
def test_forward2_protocol(stages, pair, slow_tma):
    for nkt0, nkt1 in [(0, 0), (1, 0), (1, 1), (1, 2), (3, 3), (4, 5), (6, 6), (2, 3), (5, 0)]:
        for seed in range(30):
            kp.forward2(nkt0, nkt1, seed, stages=stages, slow_tma=slow_tma, pair=pair)


@pytest.mark.parametrize("plant", ["KVEmpty0", "KVEmpty1", "KFull1", "VFull0", "PFull0", "PFull1", "SFull1",
                                   "OFinal1"])
def test_forward2_planted_mistake_is_caught(plant):
    assert (_caught(kp.forward2, plant, nkt0=4, nkt1=5) or
            _caught(kp.forward2, plant, nkt0=4, nkt1=5, slow_tma=True))


@pytest.mark.parametrize("plant", ["PairFull0", "PairFull1", "PairFull2", "PairEmpty0", "PairEmpty1",
                                   "PairEmpty2"])
def test_forward2_pair_planted_mistake_is_caught(plant):
    assert (_caught(kp.forward2, plant, nkt0=4, nkt1=5, pair=True) or
            _caught(kp.forward2, plant, nkt0=4, nkt1=5, pair=True, slow_tma=True))


def test_forward2_rescale_wait_is_implied():
    """In the two-tile forward S_t(j) is issued behind PV_t(j-1) in the same
    thread's UMMA order, so SFull_t(j) already implies that O_t holds every
    earlier product: the softmax's OStep wait before a rescale never waits
    (the model finds no hazard without it).  The kernel keeps it as a guard."""
    assert not _caught(kp.forward2, "OStep0", nkt0=4, nkt1=5)
