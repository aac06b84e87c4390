"""Compression pipeline on CPU: GPTQ beats RTN on correlated calibration inputs, codes round-trip through the
planar format, REAP selection keeps the high-saliency experts, and a quantized layer loads into the engine."""
import torch

from arcagi2_flashnext_dots3_b200.formats.planar import dequant
from arcagi2_flashnext_dots3_b200.training import compress as C


def _data(R=64, K=256, n=512, seed=0):
    g = torch.Generator().manual_seed(seed)
    W = torch.randn(R, K, generator=g) * 0.02
    basis = torch.randn(16, K, generator=g)
    x = torch.randn(n, 16, generator=g) @ basis + 0.05 * torch.randn(n, K, generator=g)  # low-rank inputs
    return W, x


def test_gptq_beats_rtn():
    W, x = _data()
    h = C.Hessian(W.shape[1])
    h.add(x)
    for bits in (4, 3, 2):
        q, s, z, dq = C.gptq(W, h.value(), bits, x.shape[0])
        qr, sr, zr = C.rtn(W, bits)
        dq_rtn = ((qr.float().view(64, 2, 128) - zr[..., None]) * sr[..., None]).view(64, 256)
        e_g, e_r = C.recon_error(W, dq, x), C.recon_error(W, dq_rtn, x)
        assert e_g < e_r, (bits, e_g, e_r)
        assert int(q.max()) <= 2 ** bits - 1


def test_codes_roundtrip_planar():
    W, x = _data()
    h = C.Hessian(256)
    h.add(x)
    q, s, z, dq = C.gptq(W, h.value(), 3, x.shape[0])
    from arcagi2_flashnext_dots3_b200.formats.planar import pack_planar
    planes = pack_planar(q.to(torch.int32), 3)
    back = dequant(planes, 3, s.half(), z.to(torch.uint8))
    assert torch.allclose(back, dq, atol=1e-6)


def test_reap_selection_and_layer_build():
    g = torch.Generator().manual_seed(3)
    E, H, I = 6, 128, 128
    experts = [(torch.randn(2 * I, H, generator=g) * (0.2 if e in (1, 4) else 0.02),
                torch.randn(H, I, generator=g) * 0.02) for e in range(E)]
    router = torch.randn(E, H, generator=g) * 0.02
    x = torch.randn(200, H, generator=g)
    logits = x @ router.t()
    sc = C.reap_scores(x, logits, experts, top_k=2)
    keep, _ = C.select_keep(sc, 3)
    assert 1 in keep and 4 in keep
    lay = C.quantize_layer(experts, router, keep, C.bits_for(3, "2:4,all:3"), x, logits, top_k=2)
    assert lay.experts == keep and [b.bits for b in lay.blobs] == [4, 4, 3]
    wgu, wd = lay.blobs[0].dense()
    assert (wgu - experts[keep[0]][0]).abs().max() < 0.5 * experts[keep[0]][0].abs().max()
