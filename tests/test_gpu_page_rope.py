"""page2d RoPE on the GPU (through the C ABI): page-bucket coordinates, the
two-axis rotary tables, their fused application and the decode coordinate
update, against the reference's outputs (golden fixture) and, on rows of
40 000 tokens, against the pinned CPU oracle.  Coordinates are integers and
compared exactly; tables within fp32 rounding (the device's sincosf against
torch's cos / sin, 2e-6) or one bf16 step; applied rotations within the
bf16 tolerance of the north star (2e-2 abs / 1e-2 rel)."""

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import page_rope as PR

pytestmark = pytest.mark.gpu

IMG, MARK = 128815, 128827


class Indexer:
    def __init__(self, span=0):
        self.image_token_id = IMG
        self.page_token_id = MARK
        self.rope_page_span = span


class Rot:
    """The attributes of DeepseekV2IndexerRotary2D the kernels read."""

    def __init__(self, inv_tok, inv_page, page_mod, dev):
        self.inv_tok = torch.from_numpy(np.asarray(inv_tok, np.float32)).to(dev)
        self.inv_page = torch.from_numpy(np.asarray(inv_page, np.float32)).to(dev)
        self.page_mod = page_mod


def t(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def bits_to_f32(a):
    return (np.asarray(a).astype(np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(torch.bfloat16)


def marker_rows(seed, B, S):
    """Seeded marker-mode documents: <PAGE> + 40-300 image tokens per prompt
    page, an instruction, then marked response pages (more of them than
    prompt pages in row 0)."""
    rng = np.random.default_rng(seed)
    out = np.full((B, S), 5, np.int64)
    for b in range(B):
        r = [0] + list(rng.integers(0, 1000, 7))
        while len(r) < S * (0.5 if b == 0 else 0.75):
            r += [MARK] + [IMG] * int(rng.integers(40, 300)) + list(rng.integers(0, 1000, int(rng.integers(0, 4))))
        r += list(rng.integers(0, 1000, 50))
        while len(r) < S:
            r += [MARK] + list(rng.integers(0, 1000, int(rng.integers(20, 200) if b == 0 else rng.integers(100, 900))))
        out[b] = np.asarray(r[:S])
    return out


def test_rope_pos_golden(cuda):
    from srswa import page_rope as P
    g = golden("page_rope")
    ids = t(g["ids"], cuda)
    S = ids.shape[1]
    for span in (0, 64):
        for tag, kl in (("full", S), ("trunc", S - 20), ("pad", S + 30)):
            ix = Indexer(span)
            tok, page = P._build_page_rope_pos(ix, ids, kl)
            np.testing.assert_array_equal(tok.cpu().numpy(), g[f"tok_sp{span}_{tag}"])
            np.testing.assert_array_equal(page.cpu().numpy(), g[f"page_sp{span}_{tag}"])
            np.testing.assert_array_equal(ix._page_rope_meta["pf_cnt"].cpu().numpy(), g[f"pfcnt_sp{span}_{tag}"])
            assert ix._page_rope_meta["n_pg"] == g[f"pfcnt_sp{span}_{tag}"].shape[1]
    assert P._build_page_rope_pos(Indexer(), t(g["bail_ids"], cuda), S) is None
    assert P._build_page_rope_pos(Indexer(), t(g["text_ids"], cuda), S) is None


def test_rope_tables_and_apply_golden(cuda):
    from srswa import page_rope as P
    g = golden("page_rope")
    tok, page = t(g["tok_sp0_full"], cuda), t(g["page_sp0_full"], cuda)
    sub = g["rot_sub"]
    for ci, pmod in ((0, 2), (1, 0)):
        rot = Rot(g[f"rot{ci}_inv_tok"], g[f"rot{ci}_inv_page"], pmod, cuda)
        for dt, tag, tol in ((torch.float32, "f32", 2e-6), (torch.bfloat16, "bf16", 4e-3)):
            cos, sin = P.rotary2d_forward(rot, torch.zeros(1, dtype=dt, device=cuda), tok, page)
            assert cos.dtype == dt and cos.shape == (3, tok.shape[1], 128)
            ref_c, ref_s = g[f"rot{ci}_cos_{tag}"], g[f"rot{ci}_sin_{tag}"]
            if tag == "bf16":
                ref_c, ref_s = bits_to_f32(ref_c), bits_to_f32(ref_s)
            got_c, got_s = cos.float().cpu().numpy(), sin.float().cpu().numpy()
            np.testing.assert_allclose(got_c[:, sub, :64], ref_c, atol=tol)
            np.testing.assert_allclose(got_s[:, sub, :64], ref_s, atol=tol)
            np.testing.assert_array_equal(got_c[..., :64], got_c[..., 64:])
    # fused application on q [B, H, P, D] (bf16), tables rounded to bf16 as in the reference
    rot = Rot(g["rot0_inv_tok"], g["rot0_inv_page"], 2, cuda)
    Pn = g["qx"].shape[2]
    for name, ref in (("qx", "qe"), ("kx", "ke")):
        x = torch.from_numpy(g[name].astype(np.int16)).view(torch.bfloat16).to(cuda)
        P.apply_rotary2d_(x, tok[:, :Pn].contiguous(), page[:, :Pn].contiguous(), rot)
        np.testing.assert_allclose(x.float().cpu().numpy(), bits_to_f32(g[ref]), atol=2e-2, rtol=1e-2)


def test_rope_decode_golden(cuda):
    from srswa import page_rope as P
    g = golden("page_rope")
    ids = t(g["ids"], cuda)
    S = ids.shape[1]

    class Ix(Indexer):     # the reference indexer's method, as srswa.dropin installs it
        _build_page_rope_pos = P._build_page_rope_pos

    class Attn:
        indexer = Ix()
        layer_idx = 0
        _main_rope_pos_2d = None
        _sparse_source_input_ids = ids

    class KV:
        pass

    attn, kv = Attn(), KV()
    tok, page = P._main_rope_coords(attn, S, kv)
    st = kv._page_rope_state[0]
    np.testing.assert_array_equal(st["page"].cpu().numpy(), g["dec_page0"])
    np.testing.assert_array_equal(st["tok"].cpu().numpy(), g["dec_tok0"])
    np.testing.assert_array_equal(st["pf_cnt"].cpu().numpy(), g["dec_pfcnt"])
    assert st["n_pg"] == int(g["dec_npg"])
    steps = t(g["dec_steps"], cuda)
    for k in range(steps.shape[1]):
        attn._sparse_source_input_ids = steps[:, k:k + 1]
        tk, pg = P._main_rope_coords(attn, 1, kv)
        np.testing.assert_array_equal(tk[:, 0].cpu().numpy(), g["dec_tok"][k])
        np.testing.assert_array_equal(pg[:, 0].cpu().numpy(), g["dec_page"][k])


@pytest.mark.parametrize("span", [0, 100])
def test_rope_long_rows_vs_oracle(cuda, span):
    """Rows of 40 000 tokens (20 scan chunks, hundreds of pages)."""
    from srswa import ops
    from srswa import page_rope as P
    B, S = 3, 40000
    ids_np = marker_rows(3 + span, B, S)
    ids = t(ids_np, cuda)
    for kl in (S, S - 999, S + 321):
        ix = Indexer(span)
        tok, page = P._build_page_rope_pos(ix, ids, kl)
        r_tok, r_page, r_pf, r_npg = PR.page_rope_pos(ids_np, IMG, MARK, kl, span)
        np.testing.assert_array_equal(page.cpu().numpy(), r_page)
        np.testing.assert_array_equal(tok.cpu().numpy(), r_tok)
        np.testing.assert_array_equal(ix._page_rope_meta["pf_cnt"].cpu().numpy(), r_pf)
        assert ix._page_rope_meta["n_pg"] == r_npg
    # tables and the fused application on [B, S, H, D] (strided view of [B, H, S, D])
    it, ip = PR.rotary2d_inv_freq(128, 10000.0, 256.0, 1, "resample")
    rot = Rot(it, ip, 2, cuda)
    cos, sin = ops.rope2d_table(tok, page, rot.inv_tok, rot.inv_page, 2)
    rc, rs = PR.rotary2d_cos_sin(r_tok, r_page, it, ip, 2)
    np.testing.assert_allclose(cos.cpu().numpy(), rc[:, :kl], atol=2e-6)
    np.testing.assert_allclose(sin.cpu().numpy(), rs[:, :kl], atol=2e-6)
    Sx = 4096
    rng = np.random.default_rng(9)
    xb = torch.from_numpy(rng.standard_normal((B, 2, Sx, 128)).astype(np.float32)).to(torch.bfloat16)
    x = xb.to(cuda)
    P.apply_rotary2d_(x, tok[:, -Sx:].contiguous(), page[:, -Sx:].contiguous(), rot)
    cb = f32_to_bf16_bits(rc[:, kl - Sx:kl]).float().numpy()
    sb = f32_to_bf16_bits(rs[:, kl - Sx:kl]).float().numpy()
    ref = PR.apply_rotary(xb.float().numpy(), cb, sb)
    np.testing.assert_allclose(x.float().cpu().numpy(), ref, atol=2e-2, rtol=1e-2)
    # fp32 activations with fp32 tables, [B, S, H, D] layout (heads_first=False)
    xf = torch.from_numpy(rng.standard_normal((B, 512, 3, 128)).astype(np.float32))
    xg = xf.to(cuda)
    P.apply_rotary2d_(xg, tok[:, :512].contiguous(), page[:, :512].contiguous(), rot, heads_first=False)
    reff = PR.apply_rotary(xf.numpy().transpose(0, 2, 1, 3), rc[:, :512], rs[:, :512]).transpose(0, 2, 1, 3)
    np.testing.assert_allclose(xg.cpu().numpy(), reff, atol=1e-4, rtol=1e-4)
    # decode: 300 tokens with markers
    st = dict(page=r_page[:, -1].copy(), tok=r_tok[:, -1].copy(), pf_cnt=r_pf, n_pg=r_npg)
    dpage, dtok = page[:, -1].clone(), tok[:, -1].clone()
    pf = ix._page_rope_meta["pf_cnt"]
    new = rng.integers(0, 1000, (B, 300))
    new[:, ::37] = MARK
    for k in range(new.shape[1]):
        ops.rope2d_decode_(t(new[:, k], cuda), MARK, dpage, dtok, pf, r_npg)
        st = PR.decode_coords_step(st, new[:, k], MARK)
        np.testing.assert_array_equal(dpage.cpu().numpy(), st["page"])
        np.testing.assert_array_equal(dtok.cpu().numpy(), st["tok"])
