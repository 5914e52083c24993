"""GPU parity of every operator against the CPU oracle, through the C ABI.

Inputs are seeded; the oracle runs on the original fp32 values, the GPU path
rounds operands to fp16 (round-to-nearest-even) and accumulates in fp32.
Tolerance: max-abs <= 1e-2 and rel-L2 <= 1e-3 (tests/_metrics.py); exact for
max pooling, concatenation and layout moves.
"""
import zlib

import numpy as np
import pytest
import torch

from oracle import oracle
from tests._metrics import assert_close

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _k():
    from lotusinfer_b200 import kernels
    return kernels


def _no_device_error():
    from lotusinfer_b200 import abi
    assert abi.device_error() == 0


def _rng(seed):
    return np.random.default_rng(seed)


def _gpu(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def _f16(a):
    """Values as the GPU sees them after fp16 rounding."""
    return np.asarray(a, np.float32).astype(np.float16).astype(np.float32)


CONV_CASES = [
    # id, n, c, h, w, cout, k, stride, pad, act, residual
    ("cfg1_64x56x56_3x3_relu", 1, 64, 56, 56, 64, 3, 1, 1, 1, False),
    ("stem_7x7_s2_cin3", 2, 3, 64, 64, 64, 7, 2, 3, 1, False),
    ("ref_test_7x7_s2_cout17", 1, 3, 131, 131, 17, 7, 2, 1, 0, False),
    ("3x3_s2_64to128", 2, 64, 28, 28, 128, 3, 2, 1, 1, False),
    ("1x1_s2_128to256", 2, 128, 14, 14, 256, 1, 2, 0, 0, False),
    ("3x3_residual_relu", 2, 128, 14, 14, 128, 3, 1, 1, 1, True),
    ("3x3_512_k4608", 1, 512, 7, 7, 512, 3, 1, 1, 1, True),
    ("cin96_general_path", 1, 96, 12, 12, 64, 3, 1, 1, 2, False),
    ("m_tail_100px", 1, 64, 10, 10, 64, 3, 1, 1, 0, False),
    ("unet_32to64", 1, 32, 40, 40, 64, 3, 1, 1, 1, False),
    ("unet_1x1_sigmoid_cout1", 2, 32, 16, 16, 1, 1, 1, 0, 2, False),
    ("alexnet_11x11_s4", 1, 3, 63, 63, 64, 11, 4, 2, 1, False),
    ("5x5_cout192", 1, 64, 13, 13, 192, 5, 1, 2, 1, False),
    # stride-1 layers with 16/32/64 channels and weights that fit in shared
    # memory run the resident-weight halo path (32/64/128-byte swizzled rows)
    ("halo_s2d_stem_like_cin12_4x4", 2, 12, 35, 35, 64, 4, 1, 0, 1, False),
    ("halo_cin16_cout40", 2, 16, 30, 30, 40, 3, 1, 1, 0, False),
    ("halo_stage1_residual", 4, 64, 56, 56, 64, 3, 1, 1, 1, True),
    ("halo_cin32_cout128_sigmoid", 1, 32, 33, 31, 128, 3, 1, 1, 2, False),
    ("halo_pad0_nonsquare", 2, 64, 34, 30, 64, 3, 1, 0, 1, False),
    # 64-channel multiples whose weights stream: one halo box per channel chunk
    ("halo4_stage2_residual", 4, 128, 28, 28, 128, 3, 1, 1, 1, True),
    ("halo4_stage3_two_ntiles", 4, 256, 14, 14, 256, 3, 1, 1, 0, False),
    ("halo4_cin192_cout96_sigmoid", 2, 192, 20, 20, 96, 3, 1, 1, 2, False),
    # Cout >= 256 on the im2col path: 256-column tiles
    ("bn256_stage3_residual", 4, 256, 14, 14, 256, 3, 1, 1, 1, True),
    ("bn256_stage4_cout512_residual", 8, 512, 7, 7, 512, 3, 1, 1, 1, True),
    ("bn256_1x1s2_cout384_partial", 4, 128, 28, 28, 384, 1, 2, 0, 0, False),
    ("bn256_3x3s2_sigmoid", 4, 128, 28, 28, 256, 3, 2, 1, 2, False),
]


@pytest.mark.parametrize("case", CONV_CASES, ids=[c[0] for c in CONV_CASES])
def test_conv2d_parity(case):
    K = _k()
    _, n, c, h, w, cout, k, s, p, act, with_res = case
    rng = _rng(zlib.crc32(case[0].encode()))
    x = rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32)
    wt = rng.normal(0, np.sqrt(2.0 / (c * k * k)), (cout, c, k, k)).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, cout).astype(np.float32)
    oh = (h + 2 * p - k) // s + 1
    ow = (w + 2 * p - k) // s + 1
    res = rng.normal(0, 1, (n, cout, oh, ow)).astype(np.float32) if with_res else None
    want = oracle.conv2d(x, wt, b, (s, s), (p, p), act, residual=res)

    xg = K.to_nhwc(_gpu(x))
    wp = K.conv2d_prepack(_gpu(wt), c)
    rg = K.to_nhwc(_gpu(res)) if with_res else None
    y = K.conv2d(xg, c, wp, _gpu(b), cout, k, s, p, act, residual=rg)
    got = K.from_nhwc(y, cout).cpu().numpy()
    assert_close(got, want, what=case[0])
    # pad channels are zero
    if y.shape[-1] != cout:
        assert torch.count_nonzero(y[..., cout:]).item() == 0
    # fp32-row output path (no residual)
    if not with_res:
        y32 = K.conv2d(xg, c, wp, _gpu(b), cout, k, s, p, act, out_f32=True)
        got32 = y32.view(n, oh, ow, cout).permute(0, 3, 1, 2).cpu().numpy()
        assert_close(got32, want, what=case[0] + "/f32")
    _no_device_error()


@pytest.mark.parametrize("amode", ["0", "1", "4"])
@pytest.mark.parametrize("case", [c for c in CONV_CASES if c[0] in (
    "cfg1_64x56x56_3x3_relu", "halo_stage1_residual", "unet_32to64", "halo_s2d_stem_like_cin12_4x4",
    "halo4_stage2_residual", "halo4_stage3_two_ntiles", "halo4_cin192_cout96_sigmoid")],
    ids=lambda c: c[0])
def test_conv2d_forced_paths(case, amode, monkeypatch):
    """Every A-staging path a layer can take gives the oracle's result: the
    cp.async gather (0), im2col TMA (1) and, for 64-channel multiples, the
    streamed-weight halo (4) next to the default choice."""
    monkeypatch.setenv("LOTUS_CONV_AMODE", amode)
    test_conv2d_parity(case)


@pytest.mark.parametrize("case", [
    # name, n, c, h, w, cout, k, pad, residual: 40-70 tiles per persistent CTA,
    # so every halo buffer, accumulator and MMA issuer is reused many times
    ("stem_s2d_like_n64", 64, 12, 115, 115, 64, 4, 0, False),
    ("stage1_residual_n256", 256, 64, 56, 56, 64, 3, 1, True),
    ("cin32_n128", 128, 32, 40, 40, 64, 3, 1, False),
    ("stage2_residual_n256", 256, 128, 28, 28, 128, 3, 1, True),
    ("stage3_n256", 256, 256, 14, 14, 256, 3, 1, False),
], ids=lambda c: c[0])
def test_conv2d_halo_many_tiles_per_cta(case, monkeypatch):
    """Full-size halo launches against the im2col / gather paths on the same
    inputs (those paths are checked against the oracle on smaller cases)."""
    K = _k()
    _, n, c, h, w, cout, k, p, with_res = case
    g = torch.Generator(device=DEV).manual_seed(zlib.crc32(case[0].encode()))
    x = K.to_nhwc(torch.rand((n, c, h, w), device=DEV, generator=g) * 2 - 1)
    wt = torch.randn((cout, c, k, k), device=DEV, generator=g) * (2.0 / (c * k * k)) ** 0.5
    b = torch.rand(cout, device=DEV, generator=g) * 0.2 - 0.1
    oh, ow = h + 2 * p - k + 1, w + 2 * p - k + 1
    res = K.to_nhwc(torch.randn((n, cout, oh, ow), device=DEV, generator=g)) if with_res else None
    wp = K.conv2d_prepack(wt, c)
    y_halo = K.conv2d(x, c, wp, b, cout, k, 1, p, 1, residual=res)
    y_again = K.conv2d(x, c, wp, b, cout, k, 1, p, 1, residual=res)
    assert torch.equal(y_halo, y_again)
    monkeypatch.setenv("LOTUS_CONV_AMODE", "1" if c % 64 == 0 else "0")
    y_ref = K.conv2d(x, c, wp, b, cout, k, 1, p, 1, residual=res)
    assert_close(K.from_nhwc(y_halo, cout).cpu().numpy(), K.from_nhwc(y_ref, cout).cpu().numpy(), what=case[0])
    if c % 64 == 0 and c > 64:
        monkeypatch.setenv("LOTUS_CONV_AMODE", "4")
        y4 = K.conv2d(x, c, wp, b, cout, k, 1, p, 1, residual=res)
        assert_close(K.from_nhwc(y4, cout).cpu().numpy(), K.from_nhwc(y_ref, cout).cpu().numpy(), what=case[0] + "/4")
    _no_device_error()


ROWS_CASES = [
    # id, n, c, h, w, cout, (kh, kw), (ph, pw), act, residual: 64-channel
    # stride-1 layers on the row-stacked kernel (forced with LOTUS_CONV_ROWS=1)
    ("rows_stage1_like_residual_odd_batch", 3, 64, 12, 12, 64, (3, 3), (1, 1), 1, True),
    ("rows_cout40_sigmoid", 2, 64, 9, 20, 40, (3, 3), (1, 1), 2, False),
    ("rows_1x1", 4, 64, 7, 7, 64, (1, 1), (0, 0), 0, False),
    ("rows_2x2_pad1", 2, 64, 6, 10, 64, (2, 2), (1, 1), 1, False),
    ("rows_pad0_one_image_a_tile_residual", 2, 64, 8, 102, 64, (3, 3), (0, 0), 1, True),  # OW = 100
    ("rows_cin60_pad_channels", 2, 60, 10, 10, 64, (3, 3), (1, 1), 1, False),
    ("rows_1x3_pad0x1", 3, 64, 5, 17, 24, (1, 3), (0, 1), 0, False),
    ("rows_3x2_pad2x0", 2, 64, 9, 9, 64, (3, 2), (2, 0), 1, True),
    # OW + kw - 1 = 64: the widest rows two images share; 65: one image a tile
    ("rows_ow62_two_images", 3, 64, 5, 62, 64, (3, 3), (1, 1), 0, False),
    ("rows_ow63_one_image", 3, 64, 5, 63, 64, (3, 3), (1, 1), 0, False),
]


@pytest.mark.parametrize("case", ROWS_CASES, ids=[c[0] for c in ROWS_CASES])
def test_conv2d_rows_kernel_parity(case, monkeypatch):
    monkeypatch.setenv("LOTUS_CONV_ROWS", "1")
    K = _k()
    _, n, c, h, w, cout, (kh, kw), (ph, pw), act, with_res = case
    rng = _rng(zlib.crc32(case[0].encode()))
    x = rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32)
    wt = rng.normal(0, np.sqrt(2.0 / (c * kh * kw)), (cout, c, kh, kw)).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, cout).astype(np.float32)
    oh, ow = h + 2 * ph - kh + 1, w + 2 * pw - kw + 1
    res = rng.normal(0, 1, (n, cout, oh, ow)).astype(np.float32) if with_res else None
    want = oracle.conv2d(x, wt, b, (1, 1), (ph, pw), act, residual=res)
    xg = K.to_nhwc(_gpu(x))
    wp = K.conv2d_prepack(_gpu(wt), c)
    rg = K.to_nhwc(_gpu(res)) if with_res else None
    y = K.conv2d(xg, c, wp, _gpu(b), cout, (kh, kw), 1, (ph, pw), act, residual=rg)
    assert_close(K.from_nhwc(y, cout).cpu().numpy(), want, what=case[0])
    if y.shape[-1] != cout:
        assert torch.count_nonzero(y[..., cout:]).item() == 0
    _no_device_error()


@pytest.mark.parametrize("with_res", [False, True], ids=["plain", "residual"])
def test_conv2d_rows_kernel_matches_general_kernel(with_res, monkeypatch):
    """ResNet-18 stage 1 at batch 256 (48 output rows per persistent CTA, so
    the A-tile ring and the TMEM ring wrap many times): the row-stacked
    kernel sums each pixel's taps in the general kernel's order, so the
    outputs are equal bit for bit."""
    K = _k()
    g = torch.Generator(device=DEV).manual_seed(5 + with_res)
    n, c, h, w = 256, 64, 56, 56
    x = K.to_nhwc(torch.rand((n, c, h, w), device=DEV, generator=g) * 2 - 1)
    wt = torch.randn((64, c, 3, 3), device=DEV, generator=g) * (2.0 / (c * 9)) ** 0.5
    b = torch.rand(64, device=DEV, generator=g) * 0.2 - 0.1
    res = K.to_nhwc(torch.randn((n, 64, h, w), device=DEV, generator=g)) if with_res else None
    wp = K.conv2d_prepack(wt, c)
    monkeypatch.setenv("LOTUS_CONV_ROWS", "1")
    y_rows = K.conv2d(x, c, wp, b, 64, 3, 1, 1, 1, residual=res)
    monkeypatch.setenv("LOTUS_CONV_ROWS", "0")
    y_gen = K.conv2d(x, c, wp, b, 64, 3, 1, 1, 1, residual=res)
    torch.cuda.synchronize()
    assert torch.equal(y_rows, y_gen)
    _no_device_error()


PAIR_CASES = [
    # id, n, c, h, w, cout, k, stride, pad, act, residual: convs over 64-channel
    # multiples on CTA pairs (forced with LOTUS_CONV_PAIR=1)
    ("pair_3x3_128_residual", 2, 128, 14, 14, 128, 3, 1, 1, 1, True),   # M = 392: odd M-tile count
    ("pair_3x3s2_64to128", 3, 64, 20, 20, 128, 3, 2, 1, 1, False),
    ("pair_1x1s2_64to256", 2, 64, 28, 28, 256, 1, 2, 0, 0, False),       # 256-column tiles
    ("pair_cout192_partial_tile", 2, 128, 9, 9, 192, 3, 1, 1, 2, False),
    ("pair_cout136_pad_channels", 1, 64, 12, 12, 136, 3, 1, 1, 1, True),
    ("pair_cin192_5x5", 1, 192, 11, 11, 128, 5, 1, 2, 1, False),
]


@pytest.mark.parametrize("case", PAIR_CASES, ids=[c[0] for c in PAIR_CASES])
def test_conv2d_pair_kernel_parity(case, monkeypatch):
    monkeypatch.setenv("LOTUS_CONV_PAIR", "1")
    _conv2d_parity_no_f32(case)


def _conv2d_parity_no_f32(case):
    K = _k()
    _, n, c, h, w, cout, k, s, p, act, with_res = case
    rng = _rng(zlib.crc32(case[0].encode()))
    x = rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32)
    wt = rng.normal(0, np.sqrt(2.0 / (c * k * k)), (cout, c, k, k)).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, cout).astype(np.float32)
    oh = (h + 2 * p - k) // s + 1
    ow = (w + 2 * p - k) // s + 1
    res = rng.normal(0, 1, (n, cout, oh, ow)).astype(np.float32) if with_res else None
    want = oracle.conv2d(x, wt, b, (s, s), (p, p), act, residual=res)
    xg = K.to_nhwc(_gpu(x))
    wp = K.conv2d_prepack(_gpu(wt), c)
    rg = K.to_nhwc(_gpu(res)) if with_res else None
    y = K.conv2d(xg, c, wp, _gpu(b), cout, k, s, p, act, residual=rg)
    assert_close(K.from_nhwc(y, cout).cpu().numpy(), want, what=case[0])
    if y.shape[-1] != cout:
        assert torch.count_nonzero(y[..., cout:]).item() == 0
    _no_device_error()


@pytest.mark.parametrize("case", [
    # name, n, c, h, w, cout, k, stride, pad, residual, pair mode: ResNet-18
    # stages 2-4 at batch 256 (many pair tiles per CTA pair: every stage ring
    # and accumulator wraps), against the general single-CTA kernel
    ("stage2_3x3_residual", 256, 128, 28, 28, 128, 3, 1, 1, True, "1"),   # 512 x 128 pair tiles
    ("stage2_3x3", 256, 128, 28, 28, 128, 3, 1, 1, False, "auto"),
    ("stage2_3x3s2", 256, 64, 56, 56, 128, 3, 2, 1, False, "auto"),
    ("stage2_1x1s2", 256, 64, 56, 56, 128, 1, 2, 0, False, "auto"),
    ("stage3_3x3", 256, 256, 14, 14, 256, 3, 1, 1, False, "auto"),
    ("stage3_1x1s2", 256, 128, 28, 28, 256, 1, 2, 0, False, "auto"),
    ("stage4_3x3_residual", 256, 512, 7, 7, 512, 3, 1, 1, True, "auto"),
    ("stage4_3x3_residual_256cols", 256, 512, 7, 7, 512, 3, 1, 1, True, "1"),
], ids=lambda c: c[0])
def test_conv2d_pair_kernel_matches_general_kernel(case, monkeypatch):
    """Each output pixel is one SM's dot products in the same K order on
    both kernels, so the outputs are equal bit for bit."""
    K = _k()
    _, n, c, h, w, cout, k, s, p, with_res, mode = case
    g = torch.Generator(device=DEV).manual_seed(zlib.crc32(case[0].encode()))
    x = K.to_nhwc(torch.rand((n, c, h, w), device=DEV, generator=g) * 2 - 1)
    wt = torch.randn((cout, c, k, k), device=DEV, generator=g) * (2.0 / (c * k * k)) ** 0.5
    b = torch.rand(cout, device=DEV, generator=g) * 0.2 - 0.1
    oh, ow = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
    res = K.to_nhwc(torch.randn((n, cout, oh, ow), device=DEV, generator=g)) if with_res else None
    wp = K.conv2d_prepack(wt, c)
    if mode == "auto":
        monkeypatch.delenv("LOTUS_CONV_PAIR", raising=False)
    else:
        monkeypatch.setenv("LOTUS_CONV_PAIR", mode)
    y_pair = K.conv2d(x, c, wp, b, cout, k, s, p, 1, residual=res)
    monkeypatch.setenv("LOTUS_CONV_PAIR", "0")
    y_gen = K.conv2d(x, c, wp, b, cout, k, s, p, 1, residual=res)
    torch.cuda.synchronize()
    assert torch.equal(y_pair, y_gen)
    _no_device_error()


@pytest.mark.parametrize("case", [
    # name, n, c, h, w, cout, k, stride, pad, residual, LOTUS_PAIR_SPLIT:
    # ResNet-18 stage 4 at batch 256 (98 pair tiles on 74 SM pairs: the last
    # 24 split over K), and, split on request although the cost model keeps
    # them whole, stage 3 (196 tiles, the last 48 split) and stage 2 (392
    # 512 x 128 tiles, the last 22 split)
    ("stage4_3x3_residual", 256, 512, 7, 7, 512, 3, 1, 1, True, None),
    ("stage4_3x3", 256, 512, 7, 7, 512, 3, 1, 1, False, None),
    ("stage4_3x3s2", 256, 256, 14, 14, 512, 3, 2, 1, False, None),
    ("stage3_3x3_residual_forced", 256, 256, 14, 14, 256, 3, 1, 1, True, "1"),
    ("stage2_3x3_residual_forced", 256, 128, 28, 28, 128, 3, 1, 1, True, "1"),
], ids=lambda c: c[0])
def test_conv2d_pair_last_wave_split(case, monkeypatch):
    """With the workspace lotus_conv2d_workspace_bytes_max asks for, the pair
    kernel splits its last wave over K and a split-K reduction finishes those
    rows: the rows of the full waves are bit-exact with the unsplit call, the
    split rows differ only by the fp32 summation order: one fp16 ulp, or
    for results near zero the fp32 rounding of a 4608-term sum (< 1e-4)."""
    from lotusinfer_b200 import abi
    monkeypatch.delenv("LOTUS_CONV_PAIR", raising=False)
    _, n, c, h, w, cout, k, s, p, with_res, split = case
    if split is None:
        monkeypatch.delenv("LOTUS_PAIR_SPLIT", raising=False)
    else:
        monkeypatch.setenv("LOTUS_PAIR_SPLIT", split)
    K = _k()
    need = K.conv2d_workspace_bytes(n, c, h, w, cout, k, s, p, 1, use_max=True)
    assert need > 0 and K.conv2d_workspace_bytes(n, c, h, w, cout, k, s, p, 1) == 0
    g = torch.Generator(device=DEV).manual_seed(zlib.crc32(case[0].encode()))
    x = K.to_nhwc(torch.rand((n, c, h, w), device=DEV, generator=g) * 2 - 1)
    wt = torch.randn((cout, c, k, k), device=DEV, generator=g) * (2.0 / (c * k * k)) ** 0.5
    b = torch.rand(cout, device=DEV, generator=g) * 0.2 - 0.1
    oh, ow = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
    res = K.to_nhwc(torch.randn((n, cout, oh, ow), device=DEV, generator=g)) if with_res else None
    wp = K.conv2d_prepack(wt, c)
    ws = torch.full((need // 4,), float("nan"), dtype=torch.float32, device=DEV)  # every read slot is written first
    launches0 = abi.launch_count()
    y_split = K.conv2d(x, c, wp, b, cout, k, s, p, 1, residual=res, workspace=ws)
    assert abi.launch_count() - launches0 == 2  # pair kernel + reduction
    y_whole = K.conv2d(x, c, wp, b, cout, k, s, p, 1, residual=res)
    torch.cuda.synchronize()
    rows_s, rows_w = y_split.reshape(-1, y_split.shape[-1]), y_whole.reshape(-1, y_whole.shape[-1])
    same = (rows_s == rows_w).all(dim=1)
    first_diff = int(torch.nonzero(~same)[0]) if not bool(same.all()) else rows_s.shape[0]
    assert first_diff >= rows_s.shape[0] // 2  # the full waves: whole rows, bit-exact
    fs, fw = rows_s.float(), rows_w.float()
    excess = (fs - fw).abs() - (torch.maximum(fs.abs(), fw.abs()) * 2.0 ** -10 + 1e-4)
    assert float(excess.max()) <= 0, f"worst excess {float(excess.max())}"
    assert not bool(torch.isnan(rows_s.float()).any())
    _no_device_error()


SPLIT_PAIR_CASES = [
    # the pair kernel with every pair tile split over K (LOTUS_PAIR_SPLIT=1
    # on launches smaller than one wave), against the oracle
    ("pair_split_3x3_128_residual", 2, 128, 14, 14, 128, 3, 1, 1, 1, True),  # 512 x 128 pair tiles
    ("pair_split_cout192_partial_tile", 2, 128, 9, 9, 192, 3, 1, 1, 2, False),
    ("pair_split_cout136_pad_channels", 1, 64, 12, 12, 136, 3, 1, 1, 1, True),
    ("pair_split_cin192_5x5", 1, 192, 11, 11, 128, 5, 1, 2, 1, False),
]


@pytest.mark.parametrize("case", SPLIT_PAIR_CASES, ids=[c[0] for c in SPLIT_PAIR_CASES])
def test_conv2d_pair_split_parity(case, monkeypatch):
    monkeypatch.setenv("LOTUS_CONV_PAIR", "1")
    monkeypatch.setenv("LOTUS_PAIR_SPLIT", "1")
    K = _k()
    _, n, c, h, w, cout, k, s, p, act, with_res = case
    need = K.conv2d_workspace_bytes(n, c, h, w, cout, k, s, p, act, use_max=True)
    assert need > 0
    rng = _rng(zlib.crc32(case[0].encode()))
    x = rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32)
    wt = rng.normal(0, np.sqrt(2.0 / (c * k * k)), (cout, c, k, k)).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, cout).astype(np.float32)
    oh = (h + 2 * p - k) // s + 1
    ow = (w + 2 * p - k) // s + 1
    res = rng.normal(0, 1, (n, cout, oh, ow)).astype(np.float32) if with_res else None
    want = oracle.conv2d(x, wt, b, (s, s), (p, p), act, residual=res)
    ws = torch.full((need // 4,), float("nan"), dtype=torch.float32, device=DEV)
    xg = K.to_nhwc(_gpu(x))
    y = K.conv2d(xg, c, K.conv2d_prepack(_gpu(wt), c), _gpu(b), cout, k, s, p, act,
                 residual=K.to_nhwc(_gpu(res)) if with_res else None, workspace=ws)
    assert_close(K.from_nhwc(y, cout).cpu().numpy(), want, what=case[0])
    if y.shape[-1] != cout:
        assert torch.count_nonzero(y[..., cout:]).item() == 0
    _no_device_error()


def test_conv2d_pair_kernel_channel_slice(monkeypatch):
    """The pair kernel writes a channel slice of a wider NHWC tensor and
    leaves the other channels untouched."""
    monkeypatch.setenv("LOTUS_CONV_PAIR", "1")
    K = _k()
    from lotusinfer_b200 import abi
    import ctypes
    g = torch.Generator(device=DEV).manual_seed(3)
    n, c, h, w, cout = 2, 128, 10, 10, 128
    x = K.to_nhwc(torch.rand((n, c, h, w), device=DEV, generator=g) * 2 - 1)
    wt = torch.randn((cout, c, 3, 3), device=DEV, generator=g) * (2.0 / (c * 9)) ** 0.5
    b = torch.rand(cout, device=DEV, generator=g) * 0.2 - 0.1
    wp = K.conv2d_prepack(wt, c)
    ref = K.conv2d(x, c, wp, b, cout, 3, 1, 1, 1)
    wide = torch.full((n, h, w, 256), 7.0, dtype=torch.float16, device=DEV)
    d = K.conv_desc(n, c, h, w, cout, 3, 1, 1, 1)
    K.check(abi.lib().lotus_conv2d_fwd_slice(K._ptr(x), K._ptr(wp), K._ptr(b), None,
                                             ctypes.c_void_p(wide.data_ptr() + 64 * 2), 256, ctypes.byref(d),
                                             None, 0, K._stream()))
    torch.cuda.synchronize()
    assert torch.equal(wide[..., 64:192], ref)
    assert bool((wide[..., :64] == 7.0).all()) and bool((wide[..., 192:] == 7.0).all())
    _no_device_error()


SPLITK_CASES = [
    # id, n, c, h, w, cout, k, stride, pad, act, residual: output grids too
    # small to fill the GPU, so the K loop splits over CTAs
    ("splitk_gather_stage3_bs1_residual", 1, 256, 14, 14, 256, 3, 1, 1, 1, True),
    ("splitk_im2col_stage2_bs1", 1, 128, 28, 28, 128, 3, 1, 1, 1, False),
    ("splitk_bn256_bs1_residual", 1, 256, 28, 28, 256, 3, 1, 1, 0, True),
    ("splitk_stage4_bs1_k4608", 1, 512, 7, 7, 512, 3, 1, 1, 1, True),
    ("splitk_cout17_sigmoid", 1, 64, 16, 16, 17, 3, 1, 1, 2, False),
]


@pytest.mark.parametrize("case", SPLITK_CASES, ids=[c[0] for c in SPLITK_CASES])
def test_conv2d_splitk_parity(case):
    """lotus_conv2d_fwd_ws: split-K partial sums + reduction (bias, residual,
    activation) against the oracle; deterministic; a too-small workspace
    runs unsplit."""
    K = _k()
    _, n, c, h, w, cout, k, s, p, act, with_res = case
    rng = _rng(zlib.crc32(case[0].encode()))
    x = rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32)
    wt = rng.normal(0, np.sqrt(2.0 / (c * k * k)), (cout, c, k, k)).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, cout).astype(np.float32)
    oh, ow = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
    res = rng.normal(0, 1, (n, cout, oh, ow)).astype(np.float32) if with_res else None
    want = oracle.conv2d(x, wt, b, (s, s), (p, p), act, residual=res)
    need = K.conv2d_workspace_bytes(n, c, h, w, cout, k, s, p, act)
    assert need > 0
    ws = torch.empty(need // 4, dtype=torch.float32, device=DEV)
    xg, wp = K.to_nhwc(_gpu(x)), K.conv2d_prepack(_gpu(wt), c)
    rg = K.to_nhwc(_gpu(res)) if with_res else None
    y = K.conv2d(xg, c, wp, _gpu(b), cout, k, s, p, act, residual=rg, workspace=ws)
    assert_close(K.from_nhwc(y, cout).cpu().numpy(), want, what=case[0])
    if y.shape[-1] != cout:
        assert torch.count_nonzero(y[..., cout:]).item() == 0
    assert torch.equal(y, K.conv2d(xg, c, wp, _gpu(b), cout, k, s, p, act, residual=rg, workspace=ws))
    small = torch.empty(need // 4 - 4, dtype=torch.float32, device=DEV)
    y_small = K.conv2d(xg, c, wp, _gpu(b), cout, k, s, p, act, residual=rg, workspace=small)
    assert_close(K.from_nhwc(y_small, cout).cpu().numpy(), want, what=case[0] + "/unsplit")
    if not with_res:
        y32 = K.conv2d(xg, c, wp, _gpu(b), cout, k, s, p, act, out_f32=True, workspace=ws)
        assert_close(y32.view(n, oh, ow, cout).permute(0, 3, 1, 2).cpu().numpy(), want, what=case[0] + "/f32")
    _no_device_error()


def test_linear_splitk_parity():
    """AlexNet-like FC at batch 32 (32 output tiles, K = 9216) through the
    split-K GEMM."""
    K = _k()
    rng = _rng(29)
    m, kk, nn = 32, 9216, 512
    wt = rng.normal(0, np.sqrt(1 / kk), (nn, kk)).astype(np.float32)
    x = rng.uniform(-1, 1, (m, kk)).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, nn).astype(np.float32)
    from lotusinfer_b200 import abi
    need = abi.lib().lotus_linear_workspace_bytes(m, kk, nn)
    assert need > 0
    ws = torch.empty(need // 4, dtype=torch.float32, device=DEV)
    wp = K.linear_prepack(_gpu(wt))
    got = K.linear(_gpu(x).half(), wp, _gpu(b), kk, nn, act=1, out_f32=True, workspace=ws).cpu().numpy()
    assert_close(got, oracle.gemm(x, wt, b, act=1), what="linear split-K")
    _no_device_error()


def test_conv2d_repeatable_and_no_bias():
    K = _k()
    rng = _rng(11)
    x = rng.normal(0, 1, (2, 64, 20, 20)).astype(np.float32)
    wt = rng.normal(0, 0.05, (128, 64, 3, 3)).astype(np.float32)
    xg, wp = K.to_nhwc(_gpu(x)), K.conv2d_prepack(_gpu(wt), 64)
    a = K.conv2d(xg, 64, wp, None, 128, 3, 1, 1)
    b = K.conv2d(xg, 64, wp, None, 128, 3, 1, 1)
    assert torch.equal(a, b)
    assert_close(K.from_nhwc(a, 128).cpu().numpy(), oracle.conv2d(x, wt, None, (1, 1), (1, 1)))


@pytest.mark.parametrize("case", [(2, 3, 224, 224, 2, 3, 112 + 3, 112 + 3), (1, 3, 224, 224, 4, 2, 57, 57),
                                  (1, 5, 17, 13, 3, 1, 7, 6),
                                  # factor 2 over 3 channels (the row-staged kernel): odd width (4-byte
                                  # loads), output past the image on both axes
                                  (2, 3, 37, 29, 2, 1, 19, 15), (1, 3, 20, 22, 2, 3, 14, 14)])
def test_space_to_depth_exact(case):
    K = _k()
    n, c, h, w, f, p, oh, ow = case
    x = _f16(_rng(13).normal(0, 1, (n, c, h, w)))
    xp = np.zeros((n, c, f * oh + f, f * ow + f), np.float32)
    hh, ww = min(h, f * oh - p), min(w, f * ow - p)
    xp[:, :, p:p + hh, p:p + ww] = x[:, :, :hh, :ww]
    want = np.zeros((n, oh, ow, K.channel_stride(c * f * f)), np.float32)
    for a in range(f):
        for b in range(f):
            want[..., (a * f + b) * c:(a * f + b + 1) * c] = xp[:, :, a:a + f * oh:f, b:b + f * ow:f].transpose(0, 2, 3, 1)
    got = K.space_to_depth(_gpu(x), f, p, (oh, ow)).float().cpu().numpy()
    np.testing.assert_array_equal(got, want)


def test_layout_round_trip_exact_for_fp16_values():
    K = _k()
    x = _f16(_rng(12).normal(0, 3, (3, 13, 9, 7)))
    back = K.from_nhwc(K.to_nhwc(_gpu(x)), 13).cpu().numpy()
    np.testing.assert_array_equal(back, x)


def test_gemm_cfg2_parity():
    K = _k()
    rng = _rng(21)
    m, nn, kk = 256, 1000, 512
    wt = rng.normal(0, np.sqrt(1 / kk), (nn, kk)).astype(np.float32)
    x = rng.uniform(-1, 1, (m, kk)).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, nn).astype(np.float32)
    want = oracle.gemm(x, wt, b)
    wp = K.linear_prepack(_gpu(wt))
    xg = _gpu(x).half()
    got = K.linear(xg, wp, _gpu(b), kk, nn, out_f32=True, force_gemm=True).cpu().numpy()
    assert_close(got, want, what="gemm cfg2")
    # relu + fp16 rows out
    got16 = K.linear(xg, wp, _gpu(b), kk, nn, act=1, out_f32=False, force_gemm=True)[:, :nn].float().cpu().numpy()
    assert_close(got16, oracle.gemm(x, wt, b, act=1), what="gemm cfg2 relu f16")
    _no_device_error()


@pytest.mark.parametrize("m", [1, 3, 8, 9, 33])
def test_linear_dispatch_gemv_and_gemm(m):
    K = _k()
    rng = _rng(22 + m)
    nn, kk = 1000, 512
    wt = rng.normal(0, np.sqrt(1 / kk), (nn, kk)).astype(np.float32)
    x = rng.uniform(-1, 1, (m, kk)).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, nn).astype(np.float32)
    wp = K.linear_prepack(_gpu(wt))
    got = K.linear(_gpu(x).half(), wp, _gpu(b), kk, nn, act=1, out_f32=True).cpu().numpy()
    assert_close(got, oracle.gemm(x, wt, b, act=1), what=f"linear m={m}")


def test_linear_flatten_permutation():
    """AlexNet's flatten of an NCHW [256,6,6] map: NHWC activations + column-permuted weights."""
    K = _k()
    rng = _rng(23)
    n, c, h, w, nn = 3, 16, 3, 3, 40
    x = rng.normal(0, 1, (n, c, h, w)).astype(np.float32)
    wt = rng.normal(0, 0.1, (nn, c * h * w)).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, nn).astype(np.float32)
    want = oracle.gemm(x.reshape(n, -1), wt, b)
    xg = K.to_nhwc(_gpu(x)).reshape(n, -1)  # (h, w, c) order
    wp = K.linear_prepack(_gpu(wt), fc_chw=(c, h, w))
    for force in (False, True):
        got = K.linear(xg, wp, _gpu(b), c * h * w, nn, out_f32=True, force_gemm=force).cpu().numpy()
        assert_close(got, want, what=f"flatten force_gemm={force}")


@pytest.mark.parametrize("shape", [(1000, 512, 1), (512, 512, 1), (4096, 9216, 1), (1000, 511, 2), (37, 96, 8)])
def test_gemv_reference_semantics_fp32(shape):
    """Fgemva semantics: fp32 W [H, W], fp32 x, fp32 y."""
    K = _k()
    hh, ww, batch = shape
    rng = _rng(hh + ww)
    wt = rng.normal(0, np.sqrt(1 / ww), (hh, ww)).astype(np.float32)
    x = rng.uniform(-1, 1, (batch, ww)).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, hh).astype(np.float32)
    got = K.gemv(_gpu(wt), _gpu(x), _gpu(b)).cpu().numpy()
    assert_close(got, oracle.gemv(wt, x, b), max_abs_tol=1e-4, rel_tol=1e-5, what=f"gemv {shape}")


@pytest.mark.parametrize("case", [
    ("resnet_3x3_s2_p1", 2, 64, 112, 112, 3, 2, 1),
    ("unet_2x2_s2", 1, 32, 64, 64, 2, 2, 0),
    ("alexnet_3x3_s2", 2, 64, 55, 55, 3, 2, 0),
    ("ref_test_9x9_s2_p4", 1, 3, 65, 65, 9, 2, 4),
    ("3x3_s2_p1_c12_odd_sizes", 3, 12, 37, 29, 3, 2, 1),
    ("3x3_s2_p1_c8_tiny", 2, 8, 2, 3, 3, 2, 1),
], ids=lambda c: c[0])
def test_maxpool_exact(case):
    K = _k()
    _, n, c, h, w, k, s, p = case
    x = _f16(_rng(31).normal(0, 1, (n, c, h, w)) - 2.0)  # negatives: -inf padding matters
    for act in (0, 1):
        want = oracle.maxpool2d(x, (k, k), (s, s), (p, p), act)
        got = K.from_nhwc(K.maxpool2d(K.to_nhwc(_gpu(x)), c, k, s, p, act), c).cpu().numpy()
        np.testing.assert_array_equal(got, _f16(want))


@pytest.mark.parametrize("case", [((2, 512, 7, 7), (1, 1)), ((1, 256, 6, 6), (6, 6)), ((1, 24, 13, 9), (6, 4)),
                                  ((1, 3, 257, 257), (64, 64)), ((3, 1000, 9, 11), (1, 1)),
                                  ((2, 2048, 5, 4), (1, 1)), ((1, 4104, 4, 4), (1, 1)), ((2, 40, 33, 17), (2, 1))])
def test_adaptive_avgpool(case):
    K = _k()
    shape, out = case
    x = _f16(_rng(41).normal(0, 1, shape))
    want = oracle.adaptive_avgpool2d(x, out)
    xg = K.to_nhwc(_gpu(x))
    got = K.from_nhwc(K.adaptive_avgpool2d(xg, shape[1], out), shape[1]).cpu().numpy()
    assert_close(got, want, what=f"aap {case}")
    got32 = K.adaptive_avgpool2d(xg, shape[1], out, out_f32=True).cpu().numpy()
    got32 = got32.reshape(shape[0], out[0], out[1], shape[1]).transpose(0, 3, 1, 2)
    assert_close(got32, want, max_abs_tol=1e-5, rel_tol=1e-6, what=f"aap f32 {case}")


def test_add_act_and_concat():
    K = _k()
    rng = _rng(51)
    a = _f16(rng.normal(0, 1, (2, 20, 9, 9)))
    b = _f16(rng.normal(0, 1, (2, 20, 9, 9)))
    got = K.from_nhwc(K.add_act(K.to_nhwc(_gpu(a)), K.to_nhwc(_gpu(b)), 20, 1), 20).cpu().numpy()
    assert_close(got, oracle.add(a, b, 1), what="add relu")
    for ca, cb in ((32, 32), (3, 5), (256, 256)):
        x1 = _f16(rng.normal(0, 1, (1, ca, 6, 7)))
        x2 = _f16(rng.normal(0, 1, (1, cb, 6, 7)))
        y = K.concat_channels(K.to_nhwc(_gpu(x1)), ca, K.to_nhwc(_gpu(x2)), cb)
        np.testing.assert_array_equal(K.from_nhwc(y, ca + cb).cpu().numpy(), oracle.concat(x1, x2))


TCONV_CASES = [
    ("unet_upconv4_512to256", 1, 512, 16, 16, 256, 2, 2, 0, 0),
    ("unet_upconv1_64to32", 2, 64, 32, 32, 32, 2, 2, 0, 0),
    ("ref_test_k2_s3_gaps", 1, 16, 64, 64, 8, 2, 3, 0, 0),
    ("overlap_k3_s2_p1_op1", 1, 24, 9, 7, 12, 3, 2, 1, 1),
    ("cout5_k2_s2", 1, 8, 5, 5, 5, 2, 2, 0, 0),
]


@pytest.mark.parametrize("case", TCONV_CASES, ids=[c[0] for c in TCONV_CASES])
def test_tconv2d_parity(case):
    K = _k()
    _, n, cin, h, w, cout, k, s, p, op = case
    rng = _rng(61)
    x = rng.uniform(-1, 1, (n, cin, h, w)).astype(np.float32)
    wt = rng.normal(0, np.sqrt(1.0 / cin), (cin, cout, k, k)).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, cout).astype(np.float32)
    for act in (0, 1):
        want = oracle.tconv2d(x, wt, b, (s, s), (p, p), (op, op), act)
        wp = K.tconv2d_prepack(_gpu(wt))
        y = K.tconv2d(K.to_nhwc(_gpu(x)), cin, wp, _gpu(b), cout, k, s, p, op, act)
        assert_close(K.from_nhwc(y, cout).cpu().numpy(), want, what=f"{case[0]} act={act}")
    _no_device_error()


ROW_CASES = [
    # id, n, c_in, h, w, cout, (kh, kw), act, pool
    # the space-to-depth ResNet stem (12 channels padded to 16, 4x4) and its 3x3/2 pool
    ("stem_s2d_bs2_pool", 2, 12, 115, 115, 64, (4, 4), 1, True),
    ("stem_s2d_bs8_pool", 8, 12, 115, 115, 64, (4, 4), 1, True),  # CTA ranges cross images
    ("stem_s2d_bs1_conv_only", 1, 12, 115, 115, 64, (4, 4), 1, False),
    # odd conv height and width (last pooled row has no row below), 40 channels (pad channels)
    ("odd_rows_cout40_pool", 3, 16, 20, 19, 40, (4, 4), 0, True),
    ("cin32_kw2_sigmoid_pool", 2, 32, 9, 30, 64, (2, 2), 2, True),
    ("cin8_kw8_kh5_conv_only", 2, 8, 16, 40, 24, (5, 8), 1, False),
    ("one_row_per_image_pool", 5, 16, 4, 50, 64, (4, 4), 1, True),  # OH = 1
    # the tallest kernel: 6-block MMA windows split at block 7 and at N = 256
    ("cin16_kw4_kh6_conv_only", 3, 16, 14, 70, 32, (6, 4), 1, False),
    ("cin16_kw4_kh6_pool", 2, 16, 23, 33, 64, (6, 4), 0, True),
    ("cin16_kw4_kh1_pool", 3, 16, 9, 60, 64, (1, 4), 1, True),
    # the widest pooled rows: 120 conv columns, 60 pooled, 15 per TMEM lane quarter
    ("ow120_pool", 2, 12, 10, 123, 64, (4, 4), 1, True),
    ("ow128_conv_only", 2, 12, 6, 131, 48, (4, 4), 0, False),
]


@pytest.mark.parametrize("case", ROW_CASES, ids=[c[0] for c in ROW_CASES])
def test_conv2d_maxpool_row_kernel(case):
    K = _k()
    _, n, c, h, w, cout, (kh, kw), act, pool = case
    rng = _rng(zlib.crc32(case[0].encode()))
    x = rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32)
    wt = rng.normal(0, np.sqrt(2.0 / (c * kh * kw)), (cout, c, kh, kw)).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, cout).astype(np.float32)
    conv = oracle.conv2d(x, wt, b, (1, 1), (0, 0), act)
    want = oracle.maxpool2d(conv, (3, 3), (2, 2), (1, 1)) if pool else conv
    xg = K.to_nhwc(_gpu(x))
    wp = K.conv2d_prepack(_gpu(wt), c)
    y = K.conv2d_maxpool(xg, c, wp, _gpu(b), cout, (kh, kw), act, pool=pool)
    got = K.from_nhwc(y, cout).cpu().numpy()
    assert_close(got, want, what=case[0])
    if y.shape[-1] != cout:
        assert torch.count_nonzero(y[..., cout:]).item() == 0
    _no_device_error()


@pytest.mark.parametrize("batch", [4, 64])
def test_conv2d_maxpool_matches_separate_conv_and_pool(batch):
    """Fused result equals the library's own conv followed by its max pool,
    bit for bit (same fp16 rounding of the conv output, max is exact); the
    row kernel's conv rows alone equal the general conv kernel's.  At batch
    64 each persistent CTA runs ~48 conv rows, so the input-row ring and the
    TMEM accumulator ring wrap several times."""
    K = _k()
    rng = _rng(11)
    x = rng.uniform(-1, 1, (batch, 12, 115, 115)).astype(np.float32)
    wt = rng.normal(0, np.sqrt(2.0 / 192), (64, 12, 4, 4)).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, 64).astype(np.float32)
    xg = K.to_nhwc(_gpu(x))
    wp = K.conv2d_prepack(_gpu(wt), 12)
    fused = K.conv2d_maxpool(xg, 12, wp, _gpu(b), 64, 4, 1)
    conv = K.conv2d(xg, 12, wp, _gpu(b), 64, 4, 1, 0, 1)
    sep = K.maxpool2d(conv, 64, 3, 2, 1)
    assert torch.equal(fused, sep)
    rows = K.conv2d_maxpool(xg, 12, wp, _gpu(b), 64, 4, 1, pool=False)
    assert torch.equal(rows, conv)
    _no_device_error()


def test_preprocess_matches_oracle_and_opencv():
    """GPU preprocessing (resize 256, RGB, /255, centre crop 224, normalise)
    against the fp32 oracle (same operation order: within fp32 rounding) and
    against OpenCV's output of the reference demo's pipeline (within one
    8-bit step)."""
    import os
    K = _k()
    d = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "preprocess_cv2.npz"))
    for name in ("down_320x240", "up_150x200"):
        img = d[name + "_bgr"]
        got = K.preprocess_bgr_u8(_gpu(img[None])).cpu().numpy()
        np.testing.assert_allclose(got, oracle.preprocess_bgr_u8(img), rtol=0, atol=2e-6)
        steps = np.abs(got[0] - d[name + "_out"]) * 255.0 * np.array(oracle.IMAGENET_STD, np.float32)[:, None, None]
        assert steps.max() <= 1.0, (name, float(steps.max()))
    # a batch of camera-sized images
    rng = _rng(5)
    imgs = rng.integers(0, 256, (8, 375, 500, 3), dtype=np.uint8)
    got = K.preprocess_bgr_u8(_gpu(imgs)).cpu().numpy()
    np.testing.assert_allclose(got, oracle.preprocess_bgr_u8(imgs), rtol=0, atol=2e-6)
    _no_device_error()
