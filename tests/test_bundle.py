"""`.gturbo` bundle loader, host side (no GPU): parsing and validation of manifest.json,
packed_experts/layout.json and the resident.bin index through the C ABI (include/gtmoe_bundle.h),
on bundles written by tests/bundle_writer.py. Cases follow the reference's format checks
(src/manifest.cpp:24-49, src/packed_experts.cpp:15-83, src/resident_index.cpp:40-97) and its
known answers in tests/test_format.cpp:28-131."""
import ctypes as C
import json
import os
import struct

import pytest

import gtmoe
import bundle_writer as bw

STRIDE = 3358720


def open_bundle(path):
    h = C.c_void_p()
    rc = gtmoe.lib().gtm_bundle_open(str(path).encode(), C.byref(h))
    return rc, h


def expect_rejected(path, fragment):
    rc, h = open_bundle(path)
    assert rc == gtmoe.ERR_INVALID, f"accepted a bad bundle (expected '{fragment}')"
    assert fragment in gtmoe.last_error(), gtmoe.last_error()


def layer_desc(h, layer, res=1 << 20, exp=1 << 30):
    L = gtmoe.Layer()
    rc = gtmoe.lib().gtm_bundle_layer_desc(h, layer, C.c_void_p(res), C.c_void_p(exp), C.byref(L))
    return rc, L


@pytest.fixture(scope="module")
def good(tmp_path_factory):
    root = tmp_path_factory.mktemp("bundle")
    plan = bw.write_bundle(str(root), num_layers=2)
    return root, plan


def test_open_reports_the_bundle(good):
    root, plan = good
    rc, h = open_bundle(root)
    assert rc == gtmoe.OK, gtmoe.last_error()
    info = gtmoe.BundleInfo()
    assert gtmoe.lib().gtm_bundle_info(h, C.byref(info)) == gtmoe.OK
    assert (info.num_layers, info.experts_per_layer, info.expert_stride) == (2, 128, STRIDE)
    assert (info.hidden, info.moe_inter, info.ffn_inter, info.top_k) == (2816, 704, 2112, 8)
    assert info.rms_norm_eps == pytest.approx(1e-6)
    assert info.resident_entries == 2 * 12 + 1
    assert info.resident_bytes == os.path.getsize(root / "resident.bin")
    assert info.resident_index_bytes % 16384 == 0
    assert info.layer_file_bytes == 128 * STRIDE
    gtmoe.lib().gtm_bundle_close(h)


def test_layer_desc_offsets_are_the_index_offsets(good):
    root, plan = good
    rc, h = open_bundle(root)
    assert rc == gtmoe.OK
    for layer in (0, 1):
        rc, L = layer_desc(h, layer)
        assert rc == gtmoe.OK, gtmoe.last_error()
        P = f"model.layers.{layer}."
        assert L.resident_dev == 1 << 20 and L.experts_dev == 1 << 30
        for q, name in ((L.router, "router.proj.weight"), (L.shared_gate, "mlp.gate_proj.weight"),
                        (L.shared_up, "mlp.up_proj.weight"), (L.shared_down, "mlp.down_proj.weight")):
            off, _, so, _, bo, _ = plan[P + name]
            assert (q.weight, q.scales, q.biases) == (off, so, bo), name
        for val, name in ((L.router_scale, "router.scale"), (L.per_expert_scale, "router.per_expert_scale"),
                          (L.pre_ffn_norm, "pre_feedforward_layernorm.weight"),
                          (L.pre_ffn_norm_2, "pre_feedforward_layernorm_2.weight"),
                          (L.post_ffn_norm_1, "post_feedforward_layernorm_1.weight"),
                          (L.post_ffn_norm_2, "post_feedforward_layernorm_2.weight"),
                          (L.post_ffn_norm, "post_feedforward_layernorm.weight"), (L.layer_scalar, "layer_scalar")):
            assert val == plan[P + name][0], name
            assert val % 16384 == 0
        # tests/test_format.cpp:96-117: raw block 3,345,408 B, stride 3,358,720, up weights at 1,115,136
        assert L.expert_stride == STRIDE
        assert (L.expert_gate.weight, L.expert_gate.scales, L.expert_gate.biases) == (0, 991232, 1053184)
        assert L.expert_up.weight == 1115136
        assert (L.expert_down.weight, L.expert_down.scales, L.expert_down.biases) == (2230272, 3221504, 3283456)
        assert 3 * L.expert_stride + L.expert_gate.weight == 3 * STRIDE
    rc, _ = layer_desc(h, 2)
    assert rc == gtmoe.ERR_INVALID and "layer 2" in gtmoe.last_error()
    gtmoe.lib().gtm_bundle_close(h)


def test_loads_validate_sizes_before_any_copy(good):
    root, _ = good
    rc, h = open_bundle(root)
    assert rc == gtmoe.OK
    L = gtmoe.lib()
    assert L.gtm_bundle_load_resident(h, C.c_void_p(4096), 16) == gtmoe.ERR_WORKSPACE
    assert L.gtm_bundle_load_experts(h, 0, 0, 2, C.c_void_p(4096), STRIDE) == gtmoe.ERR_WORKSPACE
    assert L.gtm_bundle_load_experts(h, 2, 0, 1, C.c_void_p(4096), STRIDE) == gtmoe.ERR_INVALID
    assert L.gtm_bundle_load_experts(h, 0, 120, 9, C.c_void_p(4096), 9 * STRIDE) == gtmoe.ERR_INVALID
    assert L.gtm_bundle_load_resident(h, None, 1 << 40) == gtmoe.ERR_INVALID
    L.gtm_bundle_close(h)


# ---- manifest.json (src/manifest.cpp:24-49; tests/test_format.cpp:28-47) --------------------------

def test_manifest_rejects_empty_and_wrong_magic(tmp_path):
    bw.write_bundle(str(tmp_path), num_layers=1)
    (tmp_path / "manifest.json").write_text("")
    expect_rejected(tmp_path, "manifest: empty JSON")
    (tmp_path / "manifest.json").write_text('{"magic": "NOPE"}')
    expect_rejected(tmp_path, "manifest.magic")


@pytest.mark.parametrize("edit,fragment", [
    (lambda m: m.update(versionMajor=2), "manifest.version"),
    (lambda m: m["flags"].update(someNewFlag=True), "unknown v1 flag: someNewFlag"),
    (lambda m: m.update(expertStride=3358721), "invalid dimensions or stride"),
    (lambda m: m["arch"].update(numLayers=30), "disagree with streaming metadata"),
    (lambda m: m["arch"].update(topKExperts=129), "invalid architecture values"),
    (lambda m: m.pop("expertsPerLayer"), "missing 'expertsPerLayer'"),
    (lambda m: m.update(numLayers="one"), "manifest.numLayers: expected an integer"),
])
def test_manifest_field_checks(tmp_path, edit, fragment):
    bw.write_bundle(str(tmp_path), num_layers=1, manifest_edit=edit)
    expect_rejected(tmp_path, fragment)


@pytest.mark.parametrize("text,fragment", [
    ('{"magic": "GTURBO",}', "malformed JSON"),
    ('{"magic": "GTUR', "malformed JSON"),
    ('{"magic": "GTURBO"} x', "trailing characters"),
    ('[1, 2', "malformed JSON"),
])
def test_json_reader_rejects_malformed_text(tmp_path, text, fragment):
    bw.write_bundle(str(tmp_path), num_layers=1)
    (tmp_path / "manifest.json").write_text(text)
    expect_rejected(tmp_path, fragment)


def test_json_reader_escapes_and_numbers(tmp_path):
    def edit(m):
        m["modelId"] = "gémma \"4\"\n😀"
        m["arch"]["rmsNormEps"] = 1.5e-6
        m["arch"]["extra"] = {"nested": [[1, -2.5e3, True, None], {}]}
    bw.write_bundle(str(tmp_path), num_layers=1, manifest_edit=edit)
    rc, h = open_bundle(tmp_path)
    assert rc == gtmoe.OK, gtmoe.last_error()
    info = gtmoe.BundleInfo()
    gtmoe.lib().gtm_bundle_info(h, C.byref(info))
    assert info.rms_norm_eps == pytest.approx(1.5e-6)
    gtmoe.lib().gtm_bundle_close(h)


# ---- layout.json (src/packed_experts.cpp:15-83) ------------------------------------------------

def _pop_block(name):
    return lambda lay: lay["expertBlock"].pop(name)


@pytest.mark.parametrize("edit,fragment", [
    (_pop_block("down_proj.biases"), "missing required sub-tensor 'down_proj.biases'"),
    (lambda lay: lay["expertBlock"]["up_proj.weight"].update(offset=1000), "sub-tensors overlap"),
    (lambda lay: lay["expertBlock"]["down_proj.biases"].update(size=100000), "extends past expert_stride"),
    (lambda lay: lay["layers"].pop(), "layout.layers: expected 2 entries"),
    (lambda lay: lay["layers"][1].update(layer=0), "duplicate or out-of-range layer ID 0"),
    (lambda lay: lay["layers"][1].update(file="../layer_01.bin"), "expected a plain file name"),
    (lambda lay: lay["layers"][1].update(file="sub/layer_01.bin"), "expected a plain file name"),
    (lambda lay: lay.update(expertStride=3358720 + 16384), "disagree"),
    (lambda lay: lay.update(expertStride=3358720 + 4096), "stride not a multiple of 16384"),
])
def test_layout_checks(tmp_path, edit, fragment):
    bw.write_bundle(str(tmp_path), num_layers=2, layout_edit=edit)
    expect_rejected(tmp_path, fragment)


def test_short_or_missing_layer_file(tmp_path):
    bw.write_bundle(str(tmp_path), num_layers=2)
    with open(tmp_path / "packed_experts" / "layer_01.bin", "r+b") as f:
        f.truncate(127 * STRIDE)
    expect_rejected(tmp_path, "shorter than expertsPerLayer x expertStride")
    os.remove(tmp_path / "packed_experts" / "layer_01.bin")
    expect_rejected(tmp_path, "missing file")


# ---- resident.bin index (src/resident_index.cpp:40-97; tests/test_format.cpp:119-128) ------------

def _patch(path, offset, data):
    with open(path, "r+b") as f:
        f.seek(offset)
        f.write(data)


def test_resident_header_known_answer(tmp_path):
    # tests/test_format.cpp:119-128: header {index_size 81920, resident_size 1361346560,
    # entry_count 597} little-endian at bytes 0/8/16. Here a resident.bin with exactly that header
    # (597 empty entries, the file sparse up to resident_size) goes through the decoder.
    bw.write_bundle(str(tmp_path), num_layers=1)
    index_size, resident_size, count = 81920, 1361346560, 597
    table_end = 24 + 72 * count
    region = bytearray(struct.pack("<QQQ", index_size, resident_size, count))
    names = bytearray()
    for i in range(count):
        name = f"t{i:03d}".encode()
        region += struct.pack("<IHBB", table_end + len(names), len(name), 1, 0)
        region += struct.pack("<QQ4IQQQQ", 0, 0, 0, 0, 0, 0, 0, 0, 0, 0)
        names += name
    region += names
    assert region[:24] == bytes.fromhex("0040010000000000" "0080245100000000" "5502000000000000")
    with open(tmp_path / "resident.bin", "wb") as f:
        f.write(bytes(region).ljust(index_size, b"\0"))
        f.truncate(resident_size)
    rc, h = open_bundle(tmp_path)
    assert rc == gtmoe.OK, gtmoe.last_error()
    info = gtmoe.BundleInfo()
    gtmoe.lib().gtm_bundle_info(h, C.byref(info))
    assert (info.resident_index_bytes, info.resident_bytes, info.resident_entries) == (index_size, resident_size, count)
    rc, _ = layer_desc(h, 0)   # no MoE tensors in this index
    assert rc == gtmoe.ERR_INVALID and "no tensor 'model.layers.0.router.proj.weight'" in gtmoe.last_error()
    gtmoe.lib().gtm_bundle_close(h)


def test_resident_index_checks(tmp_path):
    bw.write_bundle(str(tmp_path), num_layers=1)
    res = tmp_path / "resident.bin"
    good = res.read_bytes()
    index_size = struct.unpack_from("<Q", good, 0)[0]

    res.write_bytes(good[:10])
    expect_rejected(tmp_path, "resident.header: truncated header")
    res.write_bytes(good)
    _patch(res, 0, struct.pack("<Q", index_size + 8))
    expect_rejected(tmp_path, "truncated or unaligned index")
    res.write_bytes(good)
    _patch(res, 0, struct.pack("<Q", 32 << 20))
    expect_rejected(tmp_path, "exceeds max cap")
    res.write_bytes(good)
    _patch(res, 16, struct.pack("<Q", 100000))
    expect_rejected(tmp_path, "resident.entryTable: outside index range")
    res.write_bytes(good)
    _patch(res, 24 + 7, b"\x01")
    expect_rejected(tmp_path, "reserved byte must be zero")
    res.write_bytes(good)
    _patch(res, 24, struct.pack("<I", 8))
    expect_rejected(tmp_path, "range outside string table")
    res.write_bytes(good)
    _patch(res, 24 + 16, struct.pack("<Q", 1 << 40))
    expect_rejected(tmp_path, "past the end of resident.bin")
    res.write_bytes(good)
    rc, h = open_bundle(tmp_path)
    assert rc == gtmoe.OK
    gtmoe.lib().gtm_bundle_close(h)


def test_layer_desc_names_and_shapes(tmp_path):
    bw.write_bundle(str(tmp_path), num_layers=1)
    res = tmp_path / "resident.bin"
    good = res.read_bytes()
    index_size, _, count = struct.unpack_from("<QQQ", good, 0)
    # rename layer 0's layer_scalar -> the lookup by name fails
    for i in range(count):
        e = 24 + 72 * i
        name_off, name_len = struct.unpack_from("<IH", good, e)
        name = good[name_off:name_off + name_len].decode()
        if name == "model.layers.0.layer_scalar":
            _patch(res, name_off, b"model.layers.0.layer_scalaR")
        if name == "model.layers.0.router.proj.weight":
            router_entry = e
    rc, h = open_bundle(tmp_path)
    assert rc == gtmoe.OK
    rc, _ = layer_desc(h, 0)
    assert rc == gtmoe.ERR_INVALID and "no tensor 'model.layers.0.layer_scalar'" in gtmoe.last_error()
    gtmoe.lib().gtm_bundle_close(h)
    res.write_bytes(good)
    _patch(res, router_entry + 24, struct.pack("<I", 64))   # 64 rows: not the 128 experts
    rc, h = open_bundle(tmp_path)
    assert rc == gtmoe.OK
    rc, _ = layer_desc(h, 0)
    assert rc == gtmoe.ERR_INVALID and "router.proj.weight: expected 128 x 2816 at 8 bits" in gtmoe.last_error()
    gtmoe.lib().gtm_bundle_close(h)


def test_python_wrapper_reports_errors(tmp_path):
    from gtmoe.bundle import Bundle
    with pytest.raises(gtmoe.GtmError, match="cannot open"):
        Bundle(str(tmp_path / "nowhere"))
    bw.write_bundle(str(tmp_path), num_layers=1)
    with Bundle(str(tmp_path)) as b:
        assert b.info.num_layers == 1
