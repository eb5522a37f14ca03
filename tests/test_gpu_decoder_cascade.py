"""The device SLat decoder at cascade scale.

The reference's real shape decode grows 9,857 -> 46,537 -> 206,980 ->
909,164 -> 4,005,638 points (docs/archive/troubleshooting_history.md:400-405;
SLatDecoderModel::Impl::decode_gpu_first, src/slat_decoder.cpp:2973-3074).
Here a five-level decoder (widths 512 -> 256 -> 128 -> 64 -> 32) runs from
the 9,682-voxel shell to 4,041,472 output points with guided subdivision:
seeded keep masks (p = 0.565) stand in for the predicted logits, so the
topology is fixed and the coordinates of every level must equal the
oracle's channel-to-spatial topology bit for bit.  The features are checked
against the oracle on the first two levels (a level-truncated run the numpy
oracle finishes in seconds) and for finiteness at full scale.  The
predicted-subdivision path runs at full scale too; its topology depends on
16-bit logits near zero (the reference's own GPU and CPU paths differ there),
so only its sizes are checked.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as O
from pixal3d.cpp_b200 import workloads as WL

pytestmark = pytest.mark.gpu


def _decoder(pred_subdiv):
    from pixal3d.cpp_b200.decoder import Decoder
    w = WL.random_decoder_weights(np.random.default_rng(31), WL.CASCADE_CHANNELS, WL.CASCADE_BLOCKS,
                                  WL.CASCADE_LATENT, WL.CASCADE_OUT)
    d = Decoder(list(WL.CASCADE_CHANNELS), list(WL.CASCADE_BLOCKS), WL.CASCADE_LATENT, WL.CASCADE_OUT, w,
                pred_subdiv=pred_subdiv)
    return w, d


def _inputs():
    coords = WL.cascade_input()
    x = np.random.default_rng(32).standard_normal((coords.shape[0], WL.CASCADE_LATENT)).astype(np.float32)
    guides = WL.cascade_guides(coords.shape[0], len(WL.CASCADE_CHANNELS), seed=33)
    return coords, x, guides


def _oracle_levels(coords, x, w, guides, stop):
    """slat_decoder_forward_f32 restated (oracle.decoder_forward) up to the
    input of level `stop`: (coords, hidden)."""
    cfg = {"model_channels": list(WL.CASCADE_CHANNELS), "num_blocks": list(WL.CASCADE_BLOCKS), "norm_eps": 1e-6}
    h = O.linear(x, w["from_latent_w"], w["from_latent_b"])
    bi = 0
    for level in range(stop):
        nbr = O.neighbor_map27(coords)
        for _ in range(cfg["num_blocks"][level]):
            h = O.convnext_block(coords, h, w["blocks"][bi], cfg["norm_eps"], nbr)
            bi += 1
        coords, h, _ = O.resblock_c2s(coords, h, w["blocks"][bi], cfg["norm_eps"], cfg["model_channels"][level + 1],
                                      False, guides[level], nbr)
        bi += 1
    return coords, h


def test_decoder_cascade_guided_coords_bitexact():
    coords, x, guides = _inputs()
    w, d = _decoder(pred_subdiv=False)
    dev = torch.device("cuda", 0)
    gd = [torch.from_numpy(g).to(dev) for g in guides]
    oc, out, _ = d.run(torch.from_numpy(coords).to(dev), torch.from_numpy(x).to(dev), 1, (64, 64, 64), guides=gd)
    torch.cuda.synchronize()
    d.ctx.sync_check()
    # topology of every level: the oracle's channel-to-spatial with the same masks
    ref = coords
    sizes = [ref.shape[0]]
    for level, g in enumerate(guides):
        ref, _ = O.channel_to_spatial(ref, np.zeros((ref.shape[0], 8), np.float32), 2, g)
        sizes.append(ref.shape[0])
        got = d.run(torch.from_numpy(coords).to(dev), torch.from_numpy(x).to(dev), 1, (64, 64, 64), guides=gd,
                    stop_level=level + 1)[0] if level + 1 < len(guides) else oc
        np.testing.assert_array_equal(got.cpu().numpy(), ref, err_msg=f"level {level + 1} coordinates")
    assert sizes[-1] > 4_000_000, sizes
    assert out.shape == (sizes[-1], WL.CASCADE_OUT)
    assert bool(torch.isfinite(out).all())
    print("cascade level sizes:", sizes, flush=True)
    d.close()


def test_decoder_cascade_truncated_features_match_oracle():
    coords, x, guides = _inputs()
    w, d = _decoder(pred_subdiv=False)
    dev = torch.device("cuda", 0)
    gd = [torch.from_numpy(g).to(dev) for g in guides]
    stop = 2
    c2, h2, _ = d.run(torch.from_numpy(coords).to(dev), torch.from_numpy(x).to(dev), 1, (64, 64, 64), guides=gd,
                      stop_level=stop)
    rc, rh = _oracle_levels(coords, x, w, guides, stop)
    np.testing.assert_array_equal(c2.cpu().numpy(), rc)
    a = h2.cpu().numpy().astype(np.float64)
    e = rh.astype(np.float64)
    mx = float(np.abs(a - e).max())
    rl = float(np.linalg.norm(a - e) / np.linalg.norm(e))
    print(f"cascade level-{stop} hidden ({rc.shape[0]} x {rh.shape[1]}): max_abs {mx:.3e} rel_l2 {rl:.3e}", flush=True)
    assert rl <= 5e-3 and mx <= 2e-2 * max(1.0, float(np.abs(e).max())), (mx, rl)
    d.close()


def test_decoder_cascade_predicted_subdivision_runs():
    coords, x, _ = _inputs()
    _, d = _decoder(pred_subdiv=True)
    dev = torch.device("cuda", 0)
    oc, out, preds = d.run(torch.from_numpy(coords).to(dev), torch.from_numpy(x).to(dev), 1, (64, 64, 64))
    torch.cuda.synchronize()
    d.ctx.sync_check()
    assert len(preds) == len(WL.CASCADE_CHANNELS) - 1
    for lvl, p in enumerate(preds):
        kept = int((p > 0).sum())
        nxt = preds[lvl + 1].shape[0] if lvl + 1 < len(preds) else oc.shape[0]
        assert kept == nxt, (lvl, kept, nxt)
    assert oc.shape[0] == out.shape[0] and bool(torch.isfinite(out).all())
    d.close()
