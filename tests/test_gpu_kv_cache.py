"""A2 KV cache on the device, through the C-ABI, against the reference's own
CPU cache (native/a2_kv_cache.c, compiled into oracle/_ref) driven with the
same calls: stored K/V bits, committed lengths and key-keep masks after
every transaction (appends are copies, so equality is bit for bit), the
transaction views, the +0 scrub of an abort, and the error category/code of
every rejected call.  Cached decoding is checked as in the reference's
tests/a2/test_cache_attention.c: full attention over the sequence against
one-token steps through the cache views, both against the reference's
fixture (tests/golden/a2_attention.json, case cache.n2.incremental)."""
import numpy as np
import pytest
import torch

from eshkol_transformer_b200 import k1
from eshkol_transformer_b200.kv_cache import KvCacheApi, _CudaArray, read_view
from helpers import assert_close, decode, load_golden
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

L, N, H, CAP, D = 2, 3, 2, 8, 4


@pytest.fixture(scope="module")
def apis(lib, cuda):
    ref = orc.ref()
    if ref is None:
        pytest.fail("the reference library (oracle/_ref) is missing")
    return KvCacheApi(lib), KvCacheApi(ref)


def outcome(res):
    return res[0], res[1].category, res[1].code


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32 if a.dtype == np.float32 else a.dtype)


def same_state(ours, ref, co, cr):
    ko, vo, lo, mo = ours.snapshot(co, L)
    kr, vr, lr, mr = ref.snapshot(cr, L)
    assert np.array_equal(bits(ko), bits(kr))
    assert np.array_equal(bits(vo), bits(vr))
    assert np.array_equal(lo, lr)
    assert np.array_equal(mo, mr)


def source(rng, width, device):
    k = rng.standard_normal((N, H, width, D)).astype(np.float32)
    v = rng.standard_normal((N, H, width, D)).astype(np.float32)
    if device == "cuda":
        return k, v, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda()
    return k, v, k, v


@pytest.mark.parametrize("device", ["cpu", "cuda"])
def test_transactions_match_reference_bit_for_bit(apis, device):
    ours, ref = apis
    rng = np.random.default_rng(7)
    ro, co = ours.create(L, N, H, CAP, D)[::2]
    rr, cr = ref.create(L, N, H, CAP, D)[::2]
    assert ro == rr == 0
    lengths = np.zeros(N, np.int64)
    for step in range(12):
        width = int(rng.integers(1, 4))
        room = CAP - lengths
        counts = np.minimum(rng.integers(0, width + 1, N), room).astype(np.int64)
        if counts.sum() == 0:
            if room.max() == 0:
                break
            counts[int(np.argmax(room))] = 1
        ao, bo = ours.begin(co, width, counts), ref.begin(cr, width, counts)
        assert outcome(ao) == outcome(bo) == (0, 0, 0)
        to, tr = ao[2], bo[2]
        abort = step % 4 == 3
        layers = list(rng.permutation(L))[: (1 if abort else L)]
        for layer in layers:
            k, v, ks, vs = source(rng, width, device)
            assert outcome(ours.stage(to, layer, ks, vs)) == (0, 0, 0)
            assert outcome(ref.stage(tr, layer, k, v)) == (0, 0, 0)
            # the transaction view: effective lengths, mask and the staged layer
            vo_, vr_ = ours.view_begin(to, layer), ref.view_begin(tr, layer)
            assert outcome(vo_) == outcome(vr_) == (0, 0, 0)
            (ro_, eo, ts_o), (rr_, er, ts_r) = ours.view_tensors(vo_[2]), ref.view_tensors(vr_[2])
            assert ro_ == rr_ == 0
            assert ts_o[0].device == b"cuda" and ts_r[0].device == b"cpu"
            for a, b in zip(ts_o, ts_r):
                assert tuple(a.shape[i] for i in range(a.rank)) == \
                       tuple(b.shape[i] for i in range(b.rank))
                assert a.dtype == b.dtype and a.byte_length == b.byte_length
                assert np.array_equal(bits(read_view(a)), bits(read_view(b)))
            assert outcome(ours.view_end(vo_[2])) == outcome(ref.view_end(vr_[2])) == (0, 0, 0)
        if abort:
            assert outcome(ours.abort(to)) == outcome(ref.abort(tr)) == (0, 0, 0)
        else:
            assert outcome(ours.commit(to)) == outcome(ref.commit(tr)) == (0, 0, 0)
            lengths += counts
        same_state(ours, ref, co, cr)
    ko, vo, lo, _ = ours.snapshot(co, L)
    assert np.array_equal(lo, lengths)
    assert outcome(ours.destroy(co)) == outcome(ref.destroy(cr)) == (0, 0, 0)


def test_rejected_calls_match_reference(apis):
    ours, ref = apis
    rng = np.random.default_rng(3)
    co, cr = ours.create(L, N, H, CAP, D)[2], ref.create(L, N, H, CAP, D)[2]
    # begin: width 0, negative count, count above width, beyond capacity, all zero
    for width, counts in ((0, [1, 1, 1]), (2, [-1, 1, 1]), (2, [3, 0, 0]),
                          (CAP + 1, [CAP + 1, 0, 0]), (2, [0, 0, 0])):
        a, b = ours.begin(co, width, counts), ref.begin(cr, width, counts)
        assert outcome(a) == outcome(b) and a[0] != 0, (width, counts)
    # counts of the wrong length or dtype
    a = ours.begin(co, 2, np.array([1, 1], np.int64))
    b = ref.begin(cr, 2, np.array([1, 1], np.int64))
    assert outcome(a) == outcome(b) and a[0] != 0
    # a live transaction: second begin, borrow, destroy are refused
    to, tr = ours.begin(co, 2, [1, 2, 0])[2], ref.begin(cr, 2, [1, 2, 0])[2]
    assert outcome(ours.begin(co, 1, [1, 1, 1])) == outcome(ref.begin(cr, 1, [1, 1, 1]))
    assert outcome(ours.borrow_begin(co)) == outcome(ref.borrow_begin(cr))
    assert outcome(ours.destroy(co)) == outcome(ref.destroy(cr))
    # stage: layer out of range, wrong shape, non-finite source
    k, v, _, _ = source(rng, 2, "cpu")
    assert outcome(ours.stage(to, L, k, v)) == outcome(ref.stage(tr, L, k, v))
    assert outcome(ours.stage(to, 0, k[:, :, :1], v[:, :, :1])) == \
           outcome(ref.stage(tr, 0, k[:, :, :1], v[:, :, :1]))
    bad = k.copy()
    bad[2, 1, 1, 3] = np.inf  # in the padding of row 2 (count 0): still rejected
    assert outcome(ours.stage(to, 0, bad, v)) == outcome(ref.stage(tr, 0, bad, v))
    bad_dev = torch.from_numpy(bad).cuda()
    assert outcome(ours.stage(to, 0, bad_dev, torch.from_numpy(v).cuda()))[1:] == \
           outcome(ref.stage(tr, 0, bad, v))[1:]
    # view of an unstaged layer; commit with a layer unstaged; double stage
    assert outcome(ours.view_begin(to, 1)) == outcome(ref.view_begin(tr, 1))
    assert outcome(ours.stage(to, 0, k, v)) == outcome(ref.stage(tr, 0, k, v)) == (0, 0, 0)
    assert outcome(ours.stage(to, 0, k, v)) == outcome(ref.stage(tr, 0, k, v))
    assert outcome(ours.commit(to)) == outcome(ref.commit(tr))
    # a live view blocks staging, commit and abort
    vo, vr = ours.view_begin(to, 0)[2], ref.view_begin(tr, 0)[2]
    assert outcome(ours.stage(to, 1, k, v)) == outcome(ref.stage(tr, 1, k, v))
    assert outcome(ours.commit(to)) == outcome(ref.commit(tr))
    assert outcome(ours.abort(to)) == outcome(ref.abort(tr))
    assert outcome(ours.view_end(vo)) == outcome(ref.view_end(vr)) == (0, 0, 0)
    # abort scrubs the staged layer: the cache equals the reference again
    assert outcome(ours.abort(to)) == outcome(ref.abort(tr)) == (0, 0, 0)
    same_state(ours, ref, co, cr)
    ko, vo_, _, _ = ours.snapshot(co, L)
    assert not bits(ko).any() and not bits(vo_).any()  # every element +0
    # a live borrow blocks transactions and destroy; layer out of range
    bo, br = ours.borrow_begin(co)[2], ref.borrow_begin(cr)[2]
    assert outcome(ours.begin(co, 1, [1, 1, 1])) == outcome(ref.begin(cr, 1, [1, 1, 1]))
    assert outcome(ours.destroy(co)) == outcome(ref.destroy(cr))
    assert outcome(ours.borrow_layer(bo, L)) == outcome(ref.borrow_layer(br, L))
    assert outcome(ours.borrow_end(bo)) == outcome(ref.borrow_end(br)) == (0, 0, 0)
    assert outcome(ours.destroy(co)) == outcome(ref.destroy(cr)) == (0, 0, 0)


def _device_tensor(view):
    shape = tuple(view.shape[i] for i in range(view.rank))
    typestr = {"f32": "<f4", "i64": "<i8", "bool": "|u1"}[view.dtype.decode()]
    return torch.as_tensor(_CudaArray(view.data, shape, typestr), device="cuda")


def _dispatch(lib, capability, operation, shape, inputs, outputs):
    call = k1.KernelCall(capability, operation, tuple(shape), inputs, outputs, device="cuda")
    rc, err = k1.dispatch(k1.provider(lib, "et_a2_kernel_provider_v1"), call)
    assert rc == 0, str(err)
    torch.cuda.synchronize()


def test_cached_decoding_matches_full_attention_and_reference_fixture(apis, lib):
    """The scenario of tests/a2/test_cache_attention.c on the device."""
    ours, _ = apis
    g = load_golden("a2_attention")
    T = g["tensors"]
    q, k, v = (decode(T[f"n2_cache.input.{n}"]) for n in ("q", "k", "v"))
    positions = decode(T["n2_cache.input.positions"]).astype(np.int64)
    expected = decode(T["n2_cache.output.incremental"])  # [N, token, Hq, Dh]
    n, hq, c, dh = q.shape
    hkv = k.shape[1]
    inv = torch.tensor([0.125], dtype=torch.float32, device="cuda")  # the test's inverse frequency
    pos = torch.from_numpy(positions).cuda()
    qd, kd, vd = (torch.from_numpy(np.ascontiguousarray(x)).cuda() for x in (q, k, v))
    q_rope, k_rope = torch.empty_like(qd), torch.empty_like(kd)
    _dispatch(lib, "kernel.rope", "rope.forward", qd.shape, [qd, pos, inv], [q_rope])
    _dispatch(lib, "kernel.rope", "rope.forward", kd.shape, [kd, pos, inv], [k_rope])
    full_mask = torch.tril(torch.ones(c, c, dtype=torch.uint8, device="cuda")).expand(n, c, c)
    full_mask = full_mask.contiguous()
    full = torch.empty_like(q_rope)
    _dispatch(lib, "kernel.causal-attention", "causal-attention.forward",
              (n, hq, hkv, c, c, dh), [q_rope, k_rope, vd, pos, pos, full_mask], [full])
    want = np.transpose(expected, (0, 2, 1, 3))  # [N, Hq, token, Dh]
    assert_close(full.cpu().numpy(), want, 2e-5, 2e-5, "full attention vs fixture")

    rc, err, cache = ours.create(1, n, hkv, c, dh)
    assert rc == 0, str(err)
    for token in range(c):
        rc, err, txn = ours.begin(cache, 1, [1] * n)
        assert rc == 0, str(err)
        rc, err = ours.stage(txn, 0, k_rope[:, :, token:token + 1].contiguous(),
                             vd[:, :, token:token + 1].contiguous())
        assert rc == 0, str(err)
        rc, err, view = ours.view_begin(txn, 0)
        assert rc == 0, str(err)
        rc, err, (ck, cv, lens, mask) = ours.view_tensors(view)
        assert rc == 0, str(err)
        assert np.array_equal(read_view(lens), np.full(n, token + 1))
        m = read_view(mask)
        assert np.array_equal(m, (np.arange(c)[None, :] <= token).astype(np.uint8).repeat(n, 0))
        stored = read_view(ck)
        assert not bits(stored[:, :, token + 1:]).any()  # the tail is +0
        step_mask = _device_tensor(mask).reshape(n, 1, c).contiguous()
        out = torch.empty(n, hq, 1, dh, dtype=torch.float32, device="cuda")
        _dispatch(lib, "kernel.causal-attention", "causal-attention.forward",
                  (n, hq, hkv, 1, c, dh),
                  [q_rope[:, :, token:token + 1].contiguous(), _device_tensor(ck),
                   _device_tensor(cv), pos[:, token:token + 1].contiguous(), pos, step_mask],
                  [out])
        got = out.cpu().numpy()[:, :, 0]
        assert_close(got, full.cpu().numpy()[:, :, token], 2e-6, 0.0, f"step {token} vs full")
        assert_close(got, expected[:, token], 2e-5, 0.0, f"step {token} vs fixture")
        assert ours.view_end(view)[0] == 0
        assert ours.commit(txn)[0] == 0
    assert ours.destroy(cache)[0] == 0


def test_device_sources_from_another_stream_need_no_sync(apis):
    """K/V sources written on the caller's own stream just before
    stage_layer, with no synchronisation in between: the stage must see the
    finished values (the cache orders its reads after that work)."""
    ours, ref = apis
    rng = np.random.default_rng(11)
    co, cr = ours.create(L, N, H, CAP, D)[2], ref.create(L, N, H, CAP, D)[2]
    counts = np.array([2, 1, 2], np.int64)
    to, tr = ours.begin(co, 2, counts)[2], ref.begin(cr, 2, counts)[2]
    for layer in range(L):
        k, v, kd_src, vd_src = source(rng, 2, "cuda")
        torch.cuda.synchronize()
        producer = torch.cuda.Stream()
        with torch.cuda.stream(producer):
            kd = torch.zeros_like(kd_src)
            vd = torch.zeros_like(vd_src)
            torch.cuda._sleep(50_000_000)  # the copies below land tens of ms later
            kd.copy_(kd_src)
            vd.copy_(vd_src)
        assert outcome(ours.stage(to, layer, kd, vd)) == (0, 0, 0)
        assert outcome(ref.stage(tr, layer, k, v)) == (0, 0, 0)
    assert outcome(ours.commit(to)) == outcome(ref.commit(tr)) == (0, 0, 0)
    same_state(ours, ref, co, cr)
    assert outcome(ours.destroy(co)) == outcome(ref.destroy(cr)) == (0, 0, 0)
