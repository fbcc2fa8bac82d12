"""`.gturbo` bundle loader on the GPU: a one-layer bundle of the synthetic model (written by
tests/bundle_writer.py, expert images generated on the device) is loaded into HBM through the C
ABI. The loaded bytes equal the device's synthetic images, and the MoE block run on the
bundle's GtmLayer (batched path and fused decode) is bit-identical to the same layer built by
gtm_synth_layer_desc. Also prints the load throughput (file in the page cache -> HBM)."""
import time

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import gtmoe  # noqa: E402
from gtmoe import workloads  # noqa: E402
from gtmoe.bundle import Bundle  # noqa: E402
import bundle_writer as bw  # noqa: E402

D, K = gtmoe.HIDDEN, gtmoe.TOP_K


@pytest.fixture(scope="module")
def synth():
    m = gtmoe.SynthModel(1, seed=0)
    torch.cuda.synchronize()
    return m


@pytest.fixture(scope="module")
def bundle_dir(tmp_path_factory, synth):
    root = tmp_path_factory.mktemp("gturbo")
    img = synth.experts[0].cpu().numpy()
    bw.write_bundle(str(root), num_layers=1, seed=0, expert_images=lambda layer: img)
    return root


def test_loaded_bytes_equal_the_synthetic_images(bundle_dir, synth):
    with Bundle(str(bundle_dir)) as b:
        t0 = time.perf_counter()
        experts = b.load_experts(0)
        t1 = time.perf_counter()
        b.load_experts(0, out=experts)   # staging buffers now exist
        t2 = time.perf_counter()
        resident = b.load_resident()
        t3 = time.perf_counter()
        gb = experts.numel() / 1e9
        print(f"\nload: experts {gb:.2f} GB, first call {(t1 - t0) * 1e3:.1f} ms, again {(t2 - t1) * 1e3:.1f} ms "
              f"= {gb / (t2 - t1):.1f} GB/s (page cache -> HBM); resident {resident.numel() / 1e6:.1f} MB "
              f"in {(t3 - t2) * 1e3:.1f} ms")
        assert torch.equal(experts, synth.experts[0])
        # every MoE tensor region of the synthetic layer image at its index offset
        offs, sizes, _ = bw.synth_resident_layout()
        L = b.layer_desc(0, resident, experts)
        placed = [L.router.weight, L.router.scales, L.router.biases, L.router_scale, L.per_expert_scale,
                  L.shared_gate.weight, L.shared_gate.scales, L.shared_gate.biases,
                  L.shared_up.weight, L.shared_up.scales, L.shared_up.biases,
                  L.shared_down.weight, L.shared_down.scales, L.shared_down.biases,
                  L.pre_ffn_norm, L.pre_ffn_norm_2, L.post_ffn_norm_1, L.post_ffn_norm_2, L.post_ffn_norm,
                  L.layer_scalar]
        for o_syn, size, o_bun in zip(offs, sizes, placed):
            assert torch.equal(resident[o_bun:o_bun + size], synth.resident[0][o_syn:o_syn + size])
        # a rank's slice of the experts (expert parallelism)
        part = b.load_experts(0, first=40, count=24)
        stride = b.info.expert_stride
        assert torch.equal(part, synth.experts[0][40 * stride:64 * stride])


def test_moe_block_on_the_bundle_is_bit_identical(bundle_dir, synth):
    with Bundle(str(bundle_dir)) as b:
        resident = b.load_resident()
        experts = b.load_experts(0)
        layer = b.layer_desc(0, resident, experts)
        T = 64
        x32 = torch.empty(T * D, device="cuda")
        gtmoe.synth_x(0, 0, T, x32)
        x = x32.view(T, D)
        bias = torch.from_numpy(workloads.zipf_logit_bias()).cuda()
        outs = []
        for L in (layer, synth.layers[0]):
            blk = gtmoe.TokenBlock(T)
            out = torch.empty(T, D, device="cuda")
            idx = torch.empty(T, K, dtype=torch.int32, device="cuda")
            blk(L, x, out, topk_idx=idx, logit_bias=bias)
            blk.check()
            outs.append((out.clone(), idx.clone()))
        assert torch.equal(outs[0][1], outs[1][1])
        assert torch.equal(outs[0][0], outs[1][0])
        layers = (gtmoe.Layer * 1)(layer)
        dec_out = []
        for Ls in (layers, synth.layers):
            dec = gtmoe.Decoder(Ls, 1)
            out = torch.empty(D, device="cuda")
            dec(x32[:D], out, norm_between_layers=False)
            dec.check()
            dec_out.append(out.clone())
        assert torch.equal(dec_out[0], dec_out[1])
        torch.cuda.synchronize()
