"""File-backed expert cache (stbl_cache_create_file): the reference's expert reads from the GGUF
checkpoint (stbl/model.cu:269-308), through the C ABI on the GPU.

Layers whose routed experts stay in the file must give the bits of layers holding every expert in
device memory (the copy kernel converts the file's 17-byte MXFP4 blocks into the slot layout), the
cache's decisions must equal the reference's LRU (oracle.LruExpertCache) after every call, with
more misses per call than the staging holds (reads in rounds), O_DIRECT on and off, and with the
shadow prefetch reading on its own stream.  A read that fails (injected on the host) raises status
bit 8 and leaves the cache able to read the same experts again on the next call."""

import errno

import numpy as np
import pytest
import torch

from oracle import oracle as O
from stblarge_b200 import gguf as G
from stblarge_b200 import synth
from stblarge_b200.config import CFG1_REF
from stblarge_b200.moe import MoELayer

pytestmark = pytest.mark.gpu

L_MODEL = 3


def write_model(path, cfg, n_layers):
    """A GGUF file of n_layers MoE layers with distinct experts; returns the layers' device tensors."""
    devs = [synth.device_layer(cfg, seed_base=1000 + l * cfg.n_experts) for l in range(n_layers)]
    tensors = []
    for l, dev in enumerate(devs):
        experts = []
        for m in range(3):
            codes, scales = dev["routed_w"][m].cpu().numpy(), dev["routed_s"][m].cpu().numpy()
            E, rows, kh = codes.shape
            experts.append(O.mxfp4_to_gguf(codes.reshape(E * rows, kh), scales.reshape(E * rows, -1)).reshape(E, rows, -1))
        shared = [(dev["shared_w"][m].cpu().numpy(), dev["shared_s"][m].cpu().numpy()) for m in range(3)]
        tensors += G.moe_layer_tensors(l, dev["router_w"].cpu().numpy(), dev["router_bias"].cpu().numpy(), shared, experts)
    G.write_gguf(path, G.moe_metadata(cfg, n_layers), tensors)
    return devs


@pytest.fixture(scope="module")
def model(tmp_path_factory):
    path = tmp_path_factory.mktemp("ckpt") / "model.gguf"
    devs = write_model(path, CFG1_REF, L_MODEL)
    return path, devs


def _layers(path, devs, cache, T):
    cfg = CFG1_REF
    plain = [MoELayer(cfg, devs[l], max_tokens=T) for l in range(L_MODEL)]
    cached = []
    with G.GgufFile(path) as g:
        for l in range(L_MODEL):
            cfg_g, w = G.load_moe_layer(g, l, routed=False)
            cached.append(MoELayer(cfg_g, w, max_tokens=T, cache=(cache, l)))
    return plain, cached


def _check_state(cache, lru, what):
    mp, owner = cache.state()
    emp, eowner = lru.state(L_MODEL, CFG1_REF.n_experts)
    assert np.array_equal(mp, emp), f"{what}: residency map differs"
    assert np.array_equal(owner, eowner), f"{what}: slot owners differ"
    st = cache.stats()
    assert (st["hits"], st["misses"]) == (lru.hits, lru.misses), what


@pytest.mark.parametrize("direct", [1, 0], ids=["o_direct", "buffered"])
def test_file_backed_layers_match_resident_layers_and_reference_lru(model, direct):
    path, devs = model
    cfg, S, Tmax = CFG1_REF, 10, 2
    cache = G.file_cache(path, list(range(L_MODEL)), S, readers=3, direct=direct, stage_experts=3)
    plain, cached = _layers(path, devs, cache, Tmax)
    lru = O.LruExpertCache(S)
    rng = np.random.default_rng(21 + direct)
    for call in range(14):
        l, T = int(rng.integers(L_MODEL)), int(rng.integers(1, Tmax + 1))
        x = torch.from_numpy(synth.make_x(cfg.hidden, T, seed=700 + call).view(np.int16)).cuda()
        y_plain, y = plain[l](x), cached[l](x)
        torch.cuda.synchronize()
        assert torch.equal(y.view(torch.int16), y_plain.view(torch.int16)), f"call {call}: file-backed layer differs"
        lru.call(l, cached[l].last_route()["idx"])
        _check_state(cache, lru, f"call {call}")
    assert lru.misses > S and lru.hits > 0
    fs = cache.file_stats()
    gbytes = sum(r * (k // 32) * 17 for r, k in ((cfg.inter, cfg.hidden), (cfg.inter, cfg.hidden), (cfg.hidden, cfg.inter)))
    assert fs["failed_rounds"] == 0 and fs["seconds"] > 0
    assert lru.misses * gbytes <= fs["bytes"] <= lru.misses * (gbytes + 3 * 2 * 4096)
    if not direct:
        assert not fs["direct"]
    print(f"\nfile-backed cache ({'O_DIRECT' if fs['direct'] else 'buffered'}): {lru.misses} experts read, "
          f"{fs['bytes'] / 2**20:.1f} MiB in {fs['pieces']} pieces, {fs['seconds'] * 1e3:.1f} ms")
    for layer in cached + plain:
        assert layer.status() == 0
        layer.close()
    cache.close()


def test_file_backed_shadow_prefetch(model):
    path, devs = model
    cfg, S, T, n_predict, consider = CFG1_REF, 12, 2, 4, 3
    cache = G.file_cache(path, list(range(L_MODEL)), S, readers=2, stage_experts=2)
    plain, cached = _layers(path, devs, cache, T)
    side = torch.cuda.Stream()
    for l in range(L_MODEL - 1):
        cached[l].attach_prefetch(cached[l + 1], n_predict, consider, side)
    lru = O.LruExpertCache(S)
    for step in range(4):
        x_bits = synth.make_x(cfg.hidden, T, seed=950 + step)
        x = torch.from_numpy(x_bits.view(np.int16)).cuda()
        for l in range(L_MODEL):
            y_plain, y = plain[l](x), cached[l](x)
            torch.cuda.synchronize()
            assert torch.equal(y.view(torch.int16), y_plain.view(torch.int16)), f"step {step} layer {l}"
            lru.call(l, cached[l].last_route()["idx"])
            if l + 1 < L_MODEL:
                nw = devs[l + 1]
                lg = O.router_logits(nw["router_w"].cpu().numpy(), x_bits)
                _, guess, _ = O.router_select(lg, nw["router_bias"].cpu().numpy(), n_predict, cfg.n_groups,
                                              cfg.topk_groups, cfg.score_fn, cfg.route_scale)
                lru.prefetch(l + 1, guess, consider)
            _check_state(cache, lru, f"step {step} layer {l}")
            pf = cache.prefetch_stats()
            assert (pf["prefetched"], pf["used"]) == (lru.prefetched, lru.pf_used)
    assert lru.prefetched > 0 and lru.pf_used > 0
    for layer in cached + plain:
        assert layer.status() == 0
        layer.close()
    cache.close()


def test_failed_read_raises_status_and_is_read_again(model):
    path, devs = model
    cfg, S, T = CFG1_REF, 16, 2
    cache = G.file_cache(path, list(range(L_MODEL)), S, readers=2, stage_experts=4)
    plain, cached = _layers(path, devs, cache, T)
    x0 = torch.from_numpy(synth.make_x(cfg.hidden, T, seed=31).view(np.int16)).cuda()
    x1 = torch.from_numpy(synth.make_x(cfg.hidden, T, seed=32).view(np.int16)).cuda()
    y = cached[0](x0)
    torch.cuda.synchronize()
    assert torch.equal(y.view(torch.int16), plain[0](x0).view(torch.int16))
    assert cached[0].status() == 0
    cache.inject_read_error(0, errno.EIO)  # every read from now on fails, as a pread error would
    cached[1](x1)                          # layer 1's experts are all missing
    torch.cuda.synchronize()
    assert cached[1].status() & 8, "a failed read must raise status bit 8"
    assert cache.file_stats()["failed_rounds"] >= 1
    assert "Input/output error" in cache.error()
    cache.inject_read_error(0, 0)
    y1 = cached[1](x1)  # the experts the failed call took slots for are read again
    torch.cuda.synchronize()
    assert torch.equal(y1.view(torch.int16), plain[1](x1).view(torch.int16))
    assert cached[1].status() == 0
    y0 = cached[0](x0)  # layer 0's experts were not touched by the failure
    torch.cuda.synchronize()
    assert torch.equal(y0.view(torch.int16), plain[0](x0).view(torch.int16))
    mp, owner = cache.state()
    assert sorted(int(o) for o in owner if o >= 0) == sorted(
        {int(e) for e in cached[0].last_route()["idx"].reshape(-1)} | {cfg.n_experts + int(e) for e in cached[1].last_route()["idx"].reshape(-1)})
    for layer in cached + plain:
        assert layer.status() == 0
        layer.close()
    cache.close()
