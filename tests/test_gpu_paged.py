"""Paged KV cache (the reference's planned stage-3 layout, kvasir DESIGN.md:66-70:
blocks [block, kv_head, block_size, head_dim] addressed through a per-sequence
block table).  Only addresses change, so the bar is bit-equality with the
contiguous-cache entry points on the same keys, with the blocks scattered
through a pool that also holds unused blocks of garbage."""
import numpy as np
import pytest
import torch

from gpu_util import dev, host_bits, normal16
from oracle import oracle as O

pytestmark = pytest.mark.gpu

N_Q, N_KV, HD = 32, 8, 64


@pytest.fixture(scope="module")
def g():
    from kvasir_b200 import Gpu
    return Gpu(0)


def _scatter(rng, cache, lens, max_seq, bs, extra_blocks, dtype):
    """Contiguous [n_seq, n_kv, max_seq, hd] -> (pool, block table): sequence b's
    logical block lb goes to a random physical block; other blocks hold noise."""
    n_seq = len(lens)
    max_blocks = max_seq // bs
    need = [max(1, -(-int(n) // bs)) for n in lens]
    n_blocks = sum(need) + extra_blocks
    perm = rng.permutation(n_blocks)
    pool = normal16(rng, n_blocks * N_KV * bs * HD, dtype=dtype).reshape(n_blocks, N_KV, bs, HD)
    table = np.full((n_seq, max_blocks), -1, np.int32)
    c = cache.reshape(n_seq, N_KV, max_seq, HD)
    i = 0
    for b in range(n_seq):
        for lb in range(need[b]):
            blk = int(perm[i])
            i += 1
            table[b, lb] = blk
            pool[blk] = c[b, :, lb * bs:(lb + 1) * bs]
    return pool.reshape(-1), table


@pytest.mark.parametrize("bs", [64, 128, 256])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_paged_decode_equals_contiguous(g, bs, dtype):
    rng = np.random.default_rng(70 + bs)
    lens = np.array([1, 63, 64, 1000, 2500, 256], np.int32)
    n_seq, max_seq = len(lens), 2560
    per = N_KV * max_seq * HD
    q = normal16(rng, n_seq * N_Q * HD, dtype=dtype)
    kc = normal16(rng, n_seq * per, dtype=dtype)
    vc = normal16(rng, n_seq * per, dtype=dtype)
    kpool, table = _scatter(np.random.default_rng(7), kc, lens, max_seq, bs, 5, dtype)
    vpool, table_v = _scatter(np.random.default_rng(7), vc, lens, max_seq, bs, 5, dtype)
    assert (table == table_v).all()
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float16
    ld = torch.from_numpy(lens).cuda()
    max_len = int(lens.max())
    ws = torch.empty(max(16, g.attention_decode_workspace_bytes(n_seq, max_len, N_Q, N_KV, HD)),
                     dtype=torch.uint8, device="cuda")
    want = torch.empty(n_seq * N_Q * HD, dtype=tdt, device="cuda")
    got = torch.empty_like(want)
    g.attention_decode(dev(q, dtype), N_Q * HD, dev(kc, dtype), dev(vc, dtype), per, ld, max_len,
                       N_Q, N_KV, HD, max_seq, want, N_Q * HD, 0.125, ws)
    g.attention_decode_paged(dev(q, dtype), N_Q * HD, dev(kpool, dtype), dev(vpool, dtype),
                             torch.from_numpy(table).cuda(), table.shape[1], bs, ld, max_len, N_Q,
                             N_KV, HD, got, N_Q * HD, 0.125, ws)
    assert g.device_error() == 0
    assert torch.equal(got, want)


def test_paged_decode_without_workspace_equals_contiguous(g):
    """No workspace: one chunk per (sequence, kv head), no combine pass."""
    rng = np.random.default_rng(80)
    lens = np.array([300, 17], np.int32)
    n_seq, max_seq, bs = 2, 512, 64
    per = N_KV * max_seq * HD
    q, kc, vc = (normal16(rng, n) for n in (n_seq * N_Q * HD, n_seq * per, n_seq * per))
    kpool, table = _scatter(np.random.default_rng(3), kc, lens, max_seq, bs, 2, "bf16")
    vpool, _ = _scatter(np.random.default_rng(3), vc, lens, max_seq, bs, 2, "bf16")
    ld = torch.from_numpy(lens).cuda()
    want = torch.empty(n_seq * N_Q * HD, dtype=torch.bfloat16, device="cuda")
    got = torch.empty_like(want)
    g.attention_decode(dev(q), N_Q * HD, dev(kc), dev(vc), per, ld, 300, N_Q, N_KV, HD, max_seq,
                       want, N_Q * HD)
    g.attention_decode_paged(dev(q), N_Q * HD, dev(kpool), dev(vpool),
                             torch.from_numpy(table).cuda(), table.shape[1], bs, ld, 300, N_Q,
                             N_KV, HD, got, N_Q * HD)
    assert g.device_error() == 0
    assert torch.equal(got, want)


@pytest.mark.parametrize("t", [1, 5, 700])
def test_paged_rope_append_equals_contiguous(g, t):
    """Rows rotated identically, and the blocks gathered back in table order equal
    the contiguous cache written by kvb_rope_kv_append (unwritten slots stay zero).
    t = 700 (2100 rows) takes the warp-per-row kernel, the others the CTA-per-row one."""
    rng = np.random.default_rng(90 + t)
    n_seq, max_seq, bs = 3, 1024, 64
    pos = np.array([0, 70, 200], np.int32)
    stride = (N_Q + 2 * N_KV) * HD
    qkv = normal16(rng, n_seq * t * stride)
    cos, sin = O.cos_sin_table(HD, max_seq, **O.LLAMA3_ROPE)
    c, s = torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda()
    max_blocks = max_seq // bs
    n_blocks = n_seq * max_blocks + 3
    perm = np.random.default_rng(5).permutation(n_blocks)[:n_seq * max_blocks]
    table = perm.reshape(n_seq, max_blocks).astype(np.int32)
    kpool = torch.zeros(n_blocks * N_KV * bs * HD, dtype=torch.bfloat16, device="cuda")
    vpool = torch.zeros_like(kpool)
    a = dev(qkv)
    g.rope_kv_append_paged(a, n_seq, t, torch.from_numpy(pos).cuda(), c, s, kpool, vpool,
                           torch.from_numpy(table).cuda(), max_blocks, bs, N_Q, N_KV, HD)
    assert g.device_error() == 0
    per = N_KV * max_seq * HD
    b = dev(qkv)
    kc = torch.zeros(n_seq * per, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    for i in range(n_seq):
        g.rope_kv_append(b[i * t * stride:(i + 1) * t * stride], c, s, kc[i * per:(i + 1) * per],
                         vc[i * per:(i + 1) * per], t, int(pos[i]), N_Q, N_KV, HD, max_seq)
    np.testing.assert_array_equal(host_bits(a), host_bits(b))
    for pool, cont in ((kpool, kc), (vpool, vc)):
        p = host_bits(pool).reshape(n_blocks, N_KV, bs, HD)
        gathered = np.stack([np.concatenate([p[table[i, lb]] for lb in range(max_blocks)], axis=1)
                             for i in range(n_seq)])
        np.testing.assert_array_equal(gathered.ravel(), host_bits(cont))


def test_paged_bad_block_entry_is_flagged_not_fatal(g):
    """A table entry outside the pool sets device error code 4; the append writes
    nothing for that row, attention reads zeros there, and the GPU stays usable."""
    n_seq, bs, max_blocks, n_blocks = 2, 64, 2, 4
    stride = (N_Q + 2 * N_KV) * HD
    qkv = torch.ones(n_seq * stride, dtype=torch.bfloat16, device="cuda")
    cos, sin = O.cos_sin_table(HD, 128, 10000.0, False)
    kpool = torch.zeros(n_blocks * N_KV * bs * HD, dtype=torch.bfloat16, device="cuda")
    vpool = torch.zeros_like(kpool)
    table = torch.tensor([[0, 1], [n_blocks, 3]], dtype=torch.int32, device="cuda")
    pos = torch.tensor([5, 9], dtype=torch.int32, device="cuda")
    g.device_error()  # clear
    g.rope_kv_append_paged(qkv, n_seq, 1, pos, torch.from_numpy(cos).cuda(),
                           torch.from_numpy(sin).cuda(), kpool, vpool, table, max_blocks, bs,
                           N_Q, N_KV, HD)
    assert g.device_error() & 4
    blocks = host_bits(kpool).reshape(n_blocks, N_KV, bs, HD)
    assert blocks[0].any() and not blocks[1:].any()
    q = torch.ones(n_seq * N_Q * HD, dtype=torch.bfloat16, device="cuda")
    out = torch.empty_like(q)
    lens = torch.tensor([6, 10], dtype=torch.int32, device="cuda")
    g.attention_decode_paged(q, N_Q * HD, kpool, vpool, table, max_blocks, bs, lens, 10, N_Q, N_KV,
                             HD, out, N_Q * HD)
    assert g.device_error() & 4
    assert not torch.isnan(out.float()).any()
    x = torch.ones(16, dtype=torch.bfloat16, device="cuda")
    g.add_inplace(x, x)
    assert float(x[0]) == 2.0


def test_paged_prefill_append_bad_block_entry(g):
    """Prefill-sized append (2 x 640 rows, the bulk-copy kernel) with one table entry
    outside the pool: code 4 is raised, that block's rows are not written, and every
    other row lands exactly where the contiguous append puts it."""
    rng = np.random.default_rng(31)
    n_seq, t, max_seq, bs = 2, 640, 640, 64
    max_blocks = max_seq // bs
    stride = (N_Q + 2 * N_KV) * HD
    qkv = normal16(rng, n_seq * t * stride)
    cos, sin = O.cos_sin_table(HD, max_seq, **O.LLAMA3_ROPE)
    c, s = torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda()
    n_blocks = n_seq * max_blocks
    table = np.random.default_rng(6).permutation(n_blocks).astype(np.int32).reshape(n_seq, max_blocks)
    bad_seq, bad_lb = 1, 3
    table[bad_seq, bad_lb] = n_blocks + 7
    kpool = torch.zeros(n_blocks * N_KV * bs * HD, dtype=torch.bfloat16, device="cuda")
    vpool = torch.zeros_like(kpool)
    g.device_error()  # clear
    g.rope_kv_append_paged(dev(qkv), n_seq, t, torch.zeros(n_seq, dtype=torch.int32, device="cuda"),
                           c, s, kpool, vpool, torch.from_numpy(table).cuda(), max_blocks, bs, N_Q,
                           N_KV, HD)
    assert g.device_error() & 4
    per = N_KV * max_seq * HD
    kc = torch.zeros(n_seq * per, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    g.rope_kv_append_prefill(dev(qkv), c, s, kc, vc, n_seq, t, 0, N_Q, N_KV, HD, max_seq)
    for pool, cont in ((kpool, kc), (vpool, vc)):
        p = host_bits(pool).reshape(n_blocks, N_KV, bs, HD)
        want = host_bits(cont).reshape(n_seq, N_KV, max_blocks, bs, HD)
        for b in range(n_seq):
            for lb in range(max_blocks):
                if (b, lb) != (bad_seq, bad_lb):
                    np.testing.assert_array_equal(p[table[b, lb]], want[b, :, lb])
        used = set(int(x) for x in table.ravel())
        assert not any(p[blk].any() for blk in range(n_blocks) if blk not in used)


@pytest.mark.parametrize("n_seq,t,pos0,bs", [(2, 300, 17, 32), (1, 129, 0, 64), (3, 200, 100, 128),
                                             (1, 7, 90, 32)])
def test_paged_prefill_equals_contiguous(g, n_seq, t, pos0, bs):
    """Causal prefill through the block table == kvb_attention_prefill on the same keys;
    the pool slots past each sequence's last key hold NaN, which must not leak in."""
    rng = np.random.default_rng(n_seq * 1000 + t + pos0 + bs)
    seq_len = pos0 + t
    max_blocks = -(-seq_len // bs)
    max_seq = max_blocks * bs
    stride = (N_Q + 2 * N_KV) * HD
    qkv = normal16(rng, n_seq * t * stride)
    per = N_KV * max_seq * HD
    kc = normal16(rng, n_seq * per).reshape(n_seq, N_KV, max_seq, HD)
    vc = normal16(rng, n_seq * per).reshape(n_seq, N_KV, max_seq, HD)
    nan = np.uint16(0x7FC0)
    kc[:, :, seq_len:] = nan  # the contiguous map never reads past seq_len
    vc[:, :, seq_len:] = nan
    n_blocks = n_seq * max_blocks + 2
    perm = np.random.default_rng(bs).permutation(n_blocks)
    table = perm[:n_seq * max_blocks].reshape(n_seq, max_blocks).astype(np.int32)
    kpool = normal16(rng, n_blocks * N_KV * bs * HD).reshape(n_blocks, N_KV, bs, HD)
    vpool = normal16(rng, n_blocks * N_KV * bs * HD).reshape(n_blocks, N_KV, bs, HD)
    for b in range(n_seq):
        for lb in range(max_blocks):
            kpool[table[b, lb]] = kc[b, :, lb * bs:(lb + 1) * bs]
            vpool[table[b, lb]] = vc[b, :, lb * bs:(lb + 1) * bs]
    want = torch.empty(n_seq * t * N_Q * HD, dtype=torch.bfloat16, device="cuda")
    got = torch.empty_like(want)
    g.attention_prefill(dev(qkv), dev(kc.ravel()), dev(vc.ravel()), want, n_seq, t, pos0, N_Q, N_KV,
                        HD, max_seq)
    g.attention_prefill_paged(dev(qkv), dev(kpool.ravel()), dev(vpool.ravel()),
                              torch.from_numpy(table).cuda(), max_blocks, bs, got, n_seq, t, pos0,
                              N_Q, N_KV, HD)
    assert g.device_error() == 0
    assert not torch.isnan(got.float()).any()
    assert torch.equal(got, want)


@pytest.mark.parametrize("bs", [64, 256])
def test_paged_rope_attention_decode_equals_two_launches(g, bs):
    """kvb_rope_attention_decode_paged == kvb_rope_kv_append_paged (one row per sequence at
    lens - 1) + kvb_attention_decode_paged, bit for bit: output and both pools."""
    rng = np.random.default_rng(100 + bs)
    lens = np.array([1, 64, 65, 700, 2049], np.int32)
    n_seq, max_seq = len(lens), 2560
    max_blocks = max_seq // bs
    n_blocks = n_seq * max_blocks + 3
    table = np.random.default_rng(8).permutation(n_blocks)[:n_seq * max_blocks].astype(np.int32)
    table = table.reshape(n_seq, max_blocks)
    stride = (N_Q + 2 * N_KV) * HD
    qkv = normal16(rng, n_seq * stride)
    kpool0 = normal16(rng, n_blocks * N_KV * bs * HD)
    vpool0 = normal16(rng, n_blocks * N_KV * bs * HD)
    cos, sin = O.cos_sin_table(HD, max_seq, **O.LLAMA3_ROPE)
    c, s = torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda()
    ld = torch.from_numpy(lens).cuda()
    tb = torch.from_numpy(table).cuda()
    max_len = int(lens.max())
    ws = torch.empty(max(16, g.attention_decode_workspace_bytes(n_seq, max_len, N_Q, N_KV, HD)),
                     dtype=torch.uint8, device="cuda")
    qa, ka, va = dev(qkv), dev(kpool0), dev(vpool0)
    g.rope_kv_append_paged(qa, n_seq, 1, torch.from_numpy(lens - 1).cuda(), c, s, ka, va, tb,
                           max_blocks, bs, N_Q, N_KV, HD)
    want = torch.empty(n_seq * N_Q * HD, dtype=torch.bfloat16, device="cuda")
    g.attention_decode_paged(qa, stride, ka, va, tb, max_blocks, bs, ld, max_len, N_Q, N_KV, HD,
                             want, N_Q * HD, 0.125, ws)
    qb, kb, vb = dev(qkv), dev(kpool0), dev(vpool0)
    got = torch.empty_like(want)
    g.rope_attention_decode_paged(qb, c, s, kb, vb, tb, max_blocks, bs, ld, max_len, N_Q, N_KV, HD,
                                  got, N_Q * HD, 0.125, ws)
    assert g.device_error() == 0
    assert torch.equal(got, want)
    assert torch.equal(kb, ka) and torch.equal(vb, va)
