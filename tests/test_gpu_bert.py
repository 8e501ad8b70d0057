"""Parity of the BERT encoder on the GPU, through the drop-in C ABI
(_mlir_ciface_bert_model, src/bert-base-uncased/call_bert.cpp:41-53) and the
device entry point.

FP32 path: last_hidden_state and pooler_output within 1e-4 absolute of the
golden fixtures (HF BertModel on the same seeded weights) and of the oracle.
BF16 path (the arithmetic of the B128 x S512 BF16 workload): max |diff| of the hidden states at most
BERT_BF16_RTOL times max |hidden| of the reference, every token's hidden
vector at cosine similarity >= BERT_BF16_MIN_COS, pooled outputs (tanh, in
[-1, 1]) within BERT_BF16_POOLED_ATOL."""
import numpy as np
import pytest

from helpers import bert_golden_files, load_bert_golden, load_oracle, load_pkg

pytestmark = pytest.mark.gpu
pkg = load_pkg()
B = pkg.bert
O = load_oracle()

FP32_ATOL = 1e-4
BERT_BF16_RTOL = 0.05
BERT_BF16_MIN_COS = 0.999
BERT_BF16_POOLED_ATOL = 0.05


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available(), "GPU tests need a CUDA device"
    t.cuda.set_device(0)
    return t


def _cfg(shape, dtype):
    return B.BertConfig(shape.n_layer, shape.n_embd, shape.n_head, shape.n_inner, shape.vocab_size,
                        shape.n_positions, shape.layer_norm_eps, shape.type_vocab, dtype)


def _model(shape, blob, dtype):
    B.init(_cfg(shape, dtype), 0)
    B.load_weights(blob, '{"layout": "bert-canonical-f32-v1"}')


def _bf16_check(ref_h, got_h, ref_p, got_p, label, rows=None):
    if rows is not None:
        ref_h, got_h = ref_h[rows], got_h[rows]
    scale = float(np.abs(ref_h).max())
    err = float(np.abs(got_h - ref_h).max())
    r = ref_h.reshape(-1, ref_h.shape[-1]).astype(np.float64)
    g = got_h.reshape(-1, got_h.shape[-1]).astype(np.float64)
    cos = (r * g).sum(1) / np.maximum(np.linalg.norm(r, axis=1) * np.linalg.norm(g, axis=1), 1e-30)
    perr = float(np.abs(got_p - ref_p).max()) if ref_p is not None else 0.0
    print(f"{label}: hidden max|diff| {err:.4g} (scale {scale:.3g}, rel {err / scale:.4g}), min cos {cos.min():.6f}; "
          f"pooled max|diff| {perr:.4g}")
    assert err <= BERT_BF16_RTOL * scale, (err, scale)
    assert cos.min() >= BERT_BF16_MIN_COS, cos.min()
    assert perr <= BERT_BF16_POOLED_ATOL, perr


@pytest.mark.parametrize("path", bert_golden_files(), ids=lambda p: p.split("/")[-1])
def test_fp32_matches_golden(torch, path):
    shape, z = load_bert_golden(path)
    blob = O.bert_seeded_blob(shape, int(z["seed"]), int(z["init_mode"]))
    _model(shape, blob, B.DTYPE_F32)
    hidden, pooled = B.bert_model(z["ids"], z["token_type_ids"], z["mask"])
    assert np.abs(hidden - z["hidden"]).max() <= FP32_ATOL
    assert np.abs(pooled - z["pooled"]).max() <= FP32_ATOL


@pytest.mark.parametrize("path", bert_golden_files(), ids=lambda p: p.split("/")[-1])
def test_bf16_matches_golden(torch, path):
    shape, z = load_bert_golden(path)
    blob = O.bert_seeded_blob(shape, int(z["seed"]), int(z["init_mode"]))
    _model(shape, blob, B.DTYPE_BF16)
    hidden, pooled = B.bert_model(z["ids"], z["token_type_ids"], z["mask"])
    _bf16_check(z["hidden"], hidden, z["pooled"], pooled, path.split("/")[-1])


def test_refcall_buffers_strides_and_null_token_types(torch):
    """The reference host program's call (call_bert.cpp:61-116): position buffer arange(512),
    token-type buffer zeros, ids [101 ... 102], zeros token types, all-ones mask.  A null
    token_type_ids descriptor takes the buffer's types; strided views give the same result;
    a permuted position buffer is honoured."""
    shape, z = load_bert_golden(next(p for p in bert_golden_files() if "refcall" in p))
    blob = O.bert_seeded_blob(shape, int(z["seed"]), int(z["init_mode"]))
    _model(shape, blob, B.DTYPE_F32)
    h0, p0 = B.bert_model(z["ids"], z["token_type_ids"], z["mask"])
    h1, p1 = B.bert_model(z["ids"], None, z["mask"])
    assert np.array_equal(h0, h1) and np.array_equal(p0, p1)
    wide = np.zeros((1, 24), dtype=np.int64)
    wide[0, ::2] = z["ids"][0]
    h2, p2 = B.bert_model(wide[:, ::2], np.zeros((1, 12), dtype=np.int64), np.ones((1, 12), dtype=np.int64))
    assert np.array_equal(h0, h2) and np.array_equal(p0, p2)
    assert np.abs(h0 - z["hidden"]).max() <= FP32_ATOL
    # position buffer honoured: reversed positions against the oracle
    pos = np.arange(512, dtype=np.int64)[None].copy()
    pos[0, :12] = pos[0, :12][::-1]
    h3, p3 = B.bert_model(z["ids"], z["token_type_ids"], z["mask"], position_ids=pos)
    rh, rp = O.bert_forward(shape, blob, z["ids"], z["token_type_ids"], z["mask"], position_ids=pos[0, :12])
    assert np.abs(h3 - rh).max() <= FP32_ATOL and np.abs(p3 - rp).max() <= FP32_ATOL
    assert np.abs(h3 - h0).max() > 1e-2


def test_bf16_right_padding_lengths_s512_vs_oracle(torch):
    """Config-3 mask shape at S=512: valid lengths that end inside, on and past 128-key tile
    boundaries (key tiles past the last valid key are skipped), against the oracle."""
    shape = O.BERT_BASE
    blob = O.bert_seeded_blob(shape, 1234, 0)
    _model(shape, blob, B.DTYPE_BF16)
    lens = [64, 128, 129, 300, 512]
    ids = O.token_ids(len(lens), 512, 1234, shape.vocab_size, stream=O.BERT_IDS_STREAM)
    tt = np.zeros_like(ids)
    mask = np.zeros_like(ids)
    for b, n in enumerate(lens):
        mask[b, :n] = 1
        tt[b, n // 2:n] = 1
    hidden, pooled = B.forward_host(ids, tt, mask)
    O.set_loop_threads(8)
    rh, rp = O.bert_forward(shape, blob, ids, tt, mask)
    O.set_loop_threads(1)
    _bf16_check(rh, hidden, rp, pooled, "bf16 S512 right-padded")
    # the FP32 path agrees with the oracle within 1e-4 on the same inputs (first two sequences)
    _model(shape, blob, B.DTYPE_F32)
    h32, p32 = B.forward_host(ids[:2], tt[:2], mask[:2])
    assert np.abs(h32 - rh[:2]).max() <= FP32_ATOL
    assert np.abs(p32 - rp[:2]).max() <= FP32_ATOL


def test_bf16_config3_batch_invariance(torch):
    """The BERT workload (B=128 x S=512, BF16, lengths uniform in [64, 512]) on the device entry point:
    every sequence equals the same sequence run alone, bit for bit; two are checked against
    the oracle."""
    shape = O.BERT_BASE
    blob = O.bert_seeded_blob(shape, 1234, 0)
    _model(shape, blob, B.DTYPE_BF16)
    Bn, S, d = 128, 512, shape.n_embd
    ids_h = O.token_ids(Bn, S, 1234, shape.vocab_size, stream=O.BERT_IDS_STREAM)
    lens = 64 + O.token_ids(1, Bn, 1234, 449, stream=O.BERT_IDS_STREAM + 2)[0]
    mask_h = (np.arange(S)[None, :] < lens[:, None]).astype(np.int64)
    ids, mask = torch.from_numpy(ids_h).cuda(), torch.from_numpy(mask_h).cuda()
    hidden = torch.empty(Bn, S, d, device="cuda")
    pooled = torch.empty(Bn, d, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    B.forward_device(ids.data_ptr(), None, None, mask.data_ptr(), Bn, S, hidden.data_ptr(), pooled.data_ptr(), st)
    torch.cuda.synchronize()
    assert B.status() == 0
    h1 = torch.empty(1, S, d, device="cuda")
    p1 = torch.empty(1, d, device="cuda")
    O.set_loop_threads(8)
    for b in (0, int(np.argmin(lens)), Bn - 1):
        B.forward_device(ids[b:b + 1].contiguous().data_ptr(), None, None, mask[b:b + 1].contiguous().data_ptr(), 1,
                         S, h1.data_ptr(), p1.data_ptr(), st)
        torch.cuda.synchronize()
        assert torch.equal(hidden[b:b + 1], h1) and torch.equal(pooled[b:b + 1], p1)
        if b != 0:
            rh, rp = O.bert_forward(shape, blob, ids_h[b:b + 1], None, mask_h[b:b + 1])
            _bf16_check(rh, h1.cpu().numpy(), rp, p1.cpu().numpy(), f"bf16 B128xS512 seq {b} (len {lens[b]})")
    O.set_loop_threads(1)
    assert torch.isfinite(hidden).all() and torch.isfinite(pooled).all()


def test_errors_are_reported_not_fatal(torch):
    shape = O.BERT_TINY
    blob = O.bert_seeded_blob(shape, 5, 0)
    _model(shape, blob, B.DTYPE_F32)
    with pytest.raises(pkg.Gpt2Error, match="outside"):
        B.bert_model(np.array([[1, shape.vocab_size]]))
    with pytest.raises(pkg.Gpt2Error, match="token type"):
        B.bert_model(np.array([[1, 2]]), np.array([[0, 2]]))
    with pytest.raises(pkg.Gpt2Error):
        B.bert_model(np.zeros((1, shape.n_positions + 1), dtype=np.int64))
    # out-of-range type on the device path: status word set, context usable afterwards
    ids = torch.tensor([[1, 2, 3]], device="cuda")
    tt = torch.tensor([[0, 1, 5]], device="cuda")
    out = torch.empty(1, 3, shape.n_embd, device="cuda")
    B.forward_device(ids.data_ptr(), tt.data_ptr(), None, None, 1, 3, out.data_ptr(), None,
                     torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert B.status() == 1
    assert B.status() == 0
    h, p = B.bert_model(np.array([[1, 2, 3]]))
    assert np.isfinite(h).all() and np.isfinite(p).all()
    B.shutdown()


def test_graph_replay_matches_plain_launches(torch):
    """BERT device entry point: plain, captured and replayed forwards agree bit for bit; new ids in
    the same buffer are picked up by the replay."""
    shape = O.BERT_TINY
    blob = O.bert_seeded_blob(shape, 21, 1)
    _model(shape, blob, B.DTYPE_BF16)
    Bn, S, d = 3, 50, shape.n_embd
    st = torch.cuda.current_stream().cuda_stream
    ids = torch.from_numpy(O.token_ids(Bn, S, 21, shape.vocab_size, stream=O.BERT_IDS_STREAM)).cuda()
    mask = torch.ones(Bn, S, dtype=torch.int64, device="cuda")
    mask[1, 30:] = 0
    hidden = torch.empty(Bn, S, d, device="cuda")
    pooled = torch.empty(Bn, d, device="cuda")
    got = []
    for _ in range(3):
        B.forward_device(ids.data_ptr(), None, None, mask.data_ptr(), Bn, S, hidden.data_ptr(), pooled.data_ptr(), st)
        torch.cuda.synchronize()
        got.append((hidden.clone(), pooled.clone()))
    assert all(torch.equal(got[0][0], g[0]) and torch.equal(got[0][1], g[1]) for g in got)
    ids.copy_(torch.from_numpy(O.token_ids(Bn, S, 22, shape.vocab_size, stream=O.BERT_IDS_STREAM)).cuda())
    B.forward_device(ids.data_ptr(), None, None, mask.data_ptr(), Bn, S, hidden.data_ptr(), pooled.data_ptr(), st)
    h2 = torch.empty_like(hidden)
    B.forward_device(ids.data_ptr(), None, None, mask.data_ptr(), Bn, S, h2.data_ptr(), None, st)
    torch.cuda.synchronize()
    assert torch.equal(hidden, h2) and not torch.equal(hidden, got[0][0])
    rh, rp = O.bert_forward(shape, blob, ids.cpu().numpy(), None, mask.cpu().numpy())
    _bf16_check(rh, hidden.cpu().numpy(), rp, pooled.cpu().numpy(), "bert tiny graph replay")
    assert B.status() == 0
