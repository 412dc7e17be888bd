"""ConvInteger on the GPU against the oracle's direct convolution, bit for bit (ConvIntegerTests.cs:227-297): every
geometry of the reference's tables with all four type mixes and the zero-point modes in turn, extremes, chunked
batches through caller scratch, the Whisper and ResNet layers; each with the default and the portable product."""
import numpy as np
import pytest

import og_oracle as oracle
import onegpu_cuda as og
from cases import conv_case_data, conv_problem_dict, golden

TABLE = golden()["conv_integer"]
SENTINEL = 0x5A5A5A5A
OPTIONS = {"default": None, "portable": og.Int8GemmOptions(allow_packed_dot=False)}


def _cases_edge() -> list[dict]:
    cases = []
    for sp in TABLE["spreads"]:
        for s in range(4):
            cases.append(dict(name=f"{sp['name']} s{s}", p=sp["p"], xs=bool(s & 1), ws=bool(s & 2), xz=1 - (s & 1),
                              wz=(s + 1) % 3, fill=-1, scratch=0))
    for single in TABLE["singles"]:
        pr = single["props"]
        if single["templated"]:  # the extremes: every type mix and fill
            for s in range(4):
                for fill in TABLE["fills"]:
                    cases.append(dict(name=f"extremes {fill} s{s}", p=single["p"], xs=bool(s & 1), ws=bool(s & 2),
                                      xz=int(pr["XZeroMode"]), wz=int(pr["WZeroMode"]), fill=fill, scratch=0))
        elif "ScratchImages" in pr:
            cases.append(dict(name=single["name"], p=single["p"], xs=pr.get("XSigned", False) is True,
                              ws=pr.get("WSigned", False) is True, xz=int(pr["XZeroMode"]), wz=int(pr["WZeroMode"]),
                              fill=-1, scratch=int(pr["ScratchImages"])))
    return cases


def _cases_models() -> list[dict]:
    cases = []
    for single in TABLE["singles"]:
        pr = single["props"]
        if single["templated"] or "ScratchImages" in pr:
            continue
        cases.append(dict(name=single["name"], p=single["p"], xs=pr.get("XSigned") is True,
                          ws=pr.get("WSigned") is True, xz=int(pr["XZeroMode"]), wz=int(pr["WZeroMode"]), fill=-1,
                          scratch=0))
    return cases


def run_case(device, conv, c: dict, seed: int) -> int:
    p = c["p"]
    problem = og.ConvProblem(**conv_problem_dict(p))
    x, w, xz, wz = conv_case_data(p, seed, c["xz"], c["wz"], c["fill"], oracle.bytes_)
    want = oracle.conv_integer(p, x, c["xs"], w, c["ws"], xz, wz, c["wz"] == 2).reshape(-1)
    tx, tw = (np.int8 if c["xs"] else np.uint8), (np.int8 if c["ws"] else np.uint8)
    y_init = np.full(p["offset_y"] + want.size + 2, SENTINEL, np.int32)
    bufs = [device.create_buffer(tx, x.view(tx)), device.create_buffer(tw, w.view(tw)),
            device.create_buffer(np.int32, y_init)]
    bx, bw, by = bufs
    xzo = wzo = scratch = None
    if xz is not None:
        bufs.append(device.create_buffer(tx, xz.view(tx)))
        xzo = og.Int8Operand(bufs[-1], 0)
    if wz is not None:
        bufs.append(device.create_buffer(tw, wz.view(tw)))
        wzo = og.Int8Operand(bufs[-1], 0, c["wz"] == 2)
    scratch_offset = 0
    if c["scratch"] > 0:
        scratch_offset = 8
        scratch = device.create_buffer(tx, scratch_offset + c["scratch"] * og.conv_scratch_bytes_per_image(problem))
        bufs.append(scratch)
    try:
        enc = device.begin_commands()
        conv.encode(enc, problem, bx, bw, by, xzo, wzo, scratch, scratch_offset)
        device.submit(enc)
        got = by.read()
    finally:
        for b in bufs:
            b.dispose()
    oy = p["offset_y"]
    bad = int(np.count_nonzero(got[oy:oy + want.size] != want))
    guard = np.concatenate([got[:oy], got[oy + want.size:]])
    return bad + int(np.count_nonzero(guard != SENTINEL))


def _check(device, cases):
    failures = []
    seed = 100
    for name, options in OPTIONS.items():
        conv = og.ConvIntegerKernels(device, options)
        try:
            for c in cases:
                bad = run_case(device, conv, c, seed)
                seed += 1
                if bad:
                    failures.append(f"{c['name']} [{name}, {conv.variant}]: {bad} elements differ")
        finally:
            conv.dispose()
    assert not failures, failures


@pytest.mark.gpu
def test_edge_geometries_are_bit_exact(device):
    cases = _cases_edge()
    assert len(cases) == 4 * len(TABLE["spreads"]) + 4 * len(TABLE["fills"]) + 2
    _check(device, cases)


@pytest.mark.gpu
def test_model_layers_are_bit_exact(device):
    """The Whisper-small stem and the ResNet / MobileNet layers of the reference's tests."""
    cases = _cases_models()
    assert len(cases) == 7
    _check(device, cases)


@pytest.mark.gpu
def test_warm_calls_allocate_nothing(device):
    """ConvIntegerTests.WarmCallsBuildNoBindGroups: a second identical call creates no buffers."""
    conv = og.ConvIntegerKernels(device)
    p = og.ConvProblem(1, 3, 10, 10, 4, 3, 3, pad_top=1, pad_left=1, pad_bottom=1, pad_right=1)
    x = device.create_buffer(np.uint8, np.zeros(304, np.uint8))
    w = device.create_buffer(np.int8, np.zeros(112, np.int8))
    y = device.create_buffer(np.int32, 400)
    try:
        enc = device.begin_commands()
        conv.encode(enc, p, x, w, y)
        device.submit(enc)
        device.wait_idle()
        created = conv.bind_groups_created
        enc = device.begin_commands()
        conv.encode(enc, p, x, w, y)
        device.submit(enc)
        assert y.read()[:4].tolist() == [0, 0, 0, 0]
        assert conv.bind_groups_created == created
    finally:
        for b in (x, w, y):
            b.dispose()
        conv.dispose()


def _geometry(batch, cin, h, w, cout, kh, kw, sh=1, sw=1, dh=1, dw=1, pads=(0, 0, 0, 0), groups=1, offset_x=0):
    return dict(batch=batch, cin=cin, h=h, w=w, cout=cout, kh=kh, kw=kw, stride_h=sh, stride_w=sw, dilation_h=dh,
                dilation_w=dw, pad_top=pads[0], pad_left=pads[1], pad_bottom=pads[2], pad_right=pads[3],
                groups=groups, offset_x=offset_x, offset_w=0, offset_y=0)


# The im2col pack's paths: one-dimensional rows, word gathers at width strides 1 and 2, byte gathers at other strides, planes staged
# asynchronously (every plane on a 4-byte boundary) or byte by byte, planes above 24 KB (two buffers beyond 48 KB of
# shared memory), more planes than resident CTAs (each CTA walks several), windows cut by padding at both ends.
PACK_GEOMETRIES = [
    ("1-D stride 1, wide rows", _geometry(2, 6, 1, 4000, 5, 1, 5, pads=(0, 2, 0, 2))),
    ("2-D stride 2", _geometry(1, 3, 130, 130, 4, 3, 3, sh=2, sw=2, pads=(1, 1, 1, 1))),
    ("stride 3, dilation 2, odd width", _geometry(2, 3, 5, 1001, 4, 2, 4, sh=1, sw=3, dh=2, dw=2, pads=(1, 3, 0, 1))),
    ("40000-byte planes", _geometry(1, 2, 200, 200, 4, 3, 3, sh=2, sw=2, pads=(1, 1, 1, 1))),
    ("many planes per CTA, grouped", _geometry(4, 700, 12, 12, 8, 3, 3, pads=(1, 1, 1, 1), groups=4)),
    ("unaligned planes", _geometry(2, 5, 7, 50, 6, 3, 3, pads=(1, 1, 1, 1), offset_x=3)),
    ("depthwise stride 2", _geometry(2, 16, 33, 34, 16, 3, 3, sh=2, sw=2, pads=(1, 1, 1, 1), groups=16)),
    # one-dimensional rows (the row kernel): misaligned row starts, dilation, short rows, padding on one side
    ("1-D stride 2, odd length, offset", _geometry(3, 7, 1, 999, 4, 1, 3, sw=2, pads=(0, 1, 0, 2), offset_x=1)),
    ("1-D dilation 2, right padding only", _geometry(2, 4, 1, 517, 3, 1, 5, dw=2, pads=(0, 0, 0, 3))),
    ("1-D short rows", _geometry(4, 3, 1, 13, 2, 1, 3, sw=2, pads=(0, 1, 0, 1))),
    ("1-D stride 2, dilation 4", _geometry(2, 3, 1, 300, 2, 1, 3, sw=2, dw=4, pads=(0, 4, 0, 4))),
    ("1-D grouped stride 1", _geometry(2, 12, 1, 801, 6, 1, 3, pads=(0, 1, 0, 1), groups=3)),
]


@pytest.mark.gpu
def test_pack_layouts_are_bit_exact(device):
    cases = [dict(name=name, p=p, xs=False, ws=True, xz=1, wz=2, fill=-1, scratch=0) for name, p in PACK_GEOMETRIES]
    _check(device, cases)
