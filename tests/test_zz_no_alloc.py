"""gtm_moe_decode_noalloc, the decode entry for callers that cannot allocate device memory (a
bare C/FFI host without a device allocator, or a process that forbids allocation after start-up),
checked through the C ABI against gtm_moe_decode with a caller-allocated workspace.

Both run the same kernel on the same inputs, so the test holds them to the decode tests' gates:
top-8 indices identical and outputs within 2e-3 x RMS. Two calls in a row check that the static
scratch, which keeps the previous call's contents, is left in a usable state. The file name makes
pytest collect it last; it also passes alone in a fresh process."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import gtmoe  # noqa: E402

D, K = gtmoe.HIDDEN, gtmoe.TOP_K
NL = 3
TOL = 2e-3


def rel_max(got, ref):
    ref = np.asarray(ref, np.float64)
    return float(np.abs(np.asarray(got, np.float64) - ref).max() / np.sqrt(np.mean(ref ** 2)))


def outputs():
    return {"hidden": torch.empty(D, device="cuda"), "idx": torch.empty(NL * K, dtype=torch.int32, device="cuda"),
            "w": torch.empty(NL * K, device="cuda"), "h2": torch.empty(NL * D, device="cuda")}


def test_noalloc_matches_workspace_decode_twice():
    model = gtmoe.SynthModel(NL, seed=0)
    x = torch.empty(2 * D, device="cuda")
    gtmoe.synth_x(0, 7, 2, x)
    dec = gtmoe.Decoder(model.layers, NL)
    for call in range(2):
        xin = x[call * D:(call + 1) * D]
        ref, got = outputs(), outputs()
        dec(xin, ref["hidden"], topk_idx=ref["idx"], topk_w=ref["w"], h2=ref["h2"])
        dec.check()
        gtmoe.decode_noalloc(model.layers, xin, got["hidden"], num_layers=NL, topk_idx=got["idx"], topk_w=got["w"],
                             h2=got["h2"])
        gtmoe.decode_noalloc_check()
        torch.cuda.synchronize()
        assert torch.equal(got["idx"], ref["idx"]), f"call {call}: top-k indices differ"
        np.testing.assert_allclose(got["w"].cpu().numpy(), ref["w"].cpu().numpy(), rtol=1e-5, atol=0)
        for k in ("hidden", "h2"):
            err = rel_max(got[k].cpu().numpy(), ref[k].cpu().numpy())
            assert err <= TOL, f"call {call} {k}: {err:.3e}"


def test_noalloc_rejects_bad_layer_count():
    model = gtmoe.SynthModel(1, seed=0)
    x = torch.zeros(D, device="cuda")
    out = torch.empty(D, device="cuda")
    with pytest.raises(gtmoe.GtmError):
        gtmoe.decode_noalloc(model.layers, x, out, num_layers=gtmoe.MAX_LAYERS + 1)
