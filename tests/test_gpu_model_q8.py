"""The model ends of the decode step on resident Q8 weights, against the
oracle: the embedding gather (src/oomllama.rs:508-515), the greedy pick
(src/oomllama.rs:973-976, :1000-1003; candle's argmax) and the whole-model
decode step OomLlamaModel::forward_turbo (src/oomllama.rs:504-553) chained
over several greedy steps on a reduced two-layer model.

Embedding and argmax are bit-exact.  Logits: max-abs <= 1e-4 scaled by their
magnitude where it exceeds 1 (f32 KV).  Tokens: equal to the oracle's pick
wherever the oracle's top-two margin exceeds the logit tolerance; the oracle
then follows the library's token so both stay on one sequence."""
import numpy as np
import pytest
import torch

from helpers import F32_ATOL, assert_close, make_engine

pytestmark = pytest.mark.gpu


def _q8(oracle, rows, cols, rng, scale=0.05):
    from oomllama_b200 import Q8Matrix
    w = (rng.standard_normal((rows, cols)) * scale).astype(np.float32)
    stream = oracle.q8_quantize(w)
    return Q8Matrix.from_oom_stream(stream, rows, cols, device=0), stream


@pytest.fixture(scope="module")
def eng():
    e = make_engine(2, 1, [16])
    yield e
    e.close()


@pytest.mark.parametrize("vocab,hidden", [(1000, 256), (517, 320), (64, 3584)])
def test_embed_q8_bit_exact(oracle, eng, vocab, hidden):
    rng = np.random.default_rng(vocab + hidden)
    emb, stream = _q8(oracle, vocab, hidden, rng, scale=1.0)
    ids = np.concatenate([[0, vocab - 1, 5, 5], rng.integers(0, vocab, 29)]).astype(np.int32)
    out = eng.embed_q8(emb, torch.from_numpy(ids).cuda())
    eng.sync()
    ref = oracle.embedding(stream, vocab, hidden, ids)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))


def test_embed_q8_reports_out_of_range_ids(oracle, eng):
    from oomllama_b200._lib import OomAttnError
    rng = np.random.default_rng(7)
    emb, stream = _q8(oracle, 100, 256, rng)
    ids = torch.tensor([3, 100, -1, 99], dtype=torch.int32, device="cuda")
    out = eng.embed_q8(emb, ids)
    with pytest.raises(OomAttnError) as e:
        eng.sync()
    assert e.value.code == 9
    eng.sync()
    o = out.cpu().numpy()
    ref = oracle.embedding(stream, 100, 256, [3, 99])
    assert np.array_equal(o[[0, 3]], ref) and not o[[1, 2]].any()


def _argmax_rows(n):
    rng = np.random.default_rng(11)
    rows = []
    r = rng.standard_normal(n).astype(np.float32)
    r[[17, n // 2 - 1, n // 2, n - 1]] = 9.0  # tie: lowest index (across the row's chunks for large n)
    rows.append(r)
    r = rng.standard_normal(n).astype(np.float32)
    r[[3, n // 2]] = np.nan  # NaN skipped
    rows.append(r)
    r = rng.standard_normal(n).astype(np.float32)
    r[0] = np.nan  # NaN in element 0 is never left
    rows.append(r)
    rows.append(np.full(n, -np.inf, np.float32))  # all -inf: 0
    r = np.full(n, -np.inf, np.float32)
    r[n - 223] = -1e30
    rows.append(r)
    r = rng.standard_normal(n).astype(np.float32)
    r[n - 2] = np.inf
    r[n - 1] = np.inf
    rows.append(r)
    r = np.zeros(n, np.float32)
    r[5] = -0.0
    rows.append(r)  # +0 and -0 compare equal: 0
    r = np.full(n, np.nan, np.float32)
    r[n - 1] = -5.0
    rows.append(r)  # NaN in element 0: 0, even though a number follows
    r = np.full(n, np.nan, np.float32)
    r[0] = 1.0
    rows.append(r)  # only element 0 is a number
    return np.stack(rows)


@pytest.mark.parametrize("n", [1000, 20000])
def test_argmax_edge_cases(oracle, eng, n):
    x = _argmax_rows(n)
    ids = eng.argmax(torch.from_numpy(x).cuda())
    eng.sync()
    ref = oracle.argmax(x)
    assert ids.cpu().numpy().tolist() == ref.tolist()
    assert ref.tolist() == [oracle.argmax_scan(r) for r in x]


@pytest.mark.parametrize("R,n", [(1, 1), (3, 513), (16, 152064), (2, 128256)])
def test_argmax_sizes(oracle, eng, R, n):
    rng = np.random.default_rng(R * n)
    x = rng.standard_normal((R, n)).astype(np.float32)
    x[:, rng.integers(0, n, 4)] = x.max() + 1.0  # a tie at the top of every row
    ids = eng.argmax(torch.from_numpy(x).cuda())
    eng.sync()
    assert ids.cpu().numpy().tolist() == oracle.argmax(x).tolist()


def _model(oracle, n_layers, hq, hkv, inter, vocab, seed):
    from oomllama_b200 import Q8DecoderLayer, Q8Model
    D = 128
    H = hq * D
    rng = np.random.default_rng(seed)
    dev = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    layers, ref_layers = [], []
    for _ in range(n_layers):
        mats, deq = {}, {}
        for name, (r, c) in {"q": (hq * D, H), "k": (hkv * D, H), "v": (hkv * D, H), "o": (H, hq * D),
                             "gate": (inter, H), "up": (inter, H), "down": (H, inter)}.items():
            mats[name], stream = _q8(oracle, r, c, rng)
            deq[name] = oracle.q8_dequantize(stream, r * c).reshape(r, c)
        bq, bk, bv = [(rng.standard_normal(n) * 0.1).astype(np.float32) for n in (hq * D, hkv * D, hkv * D)]
        n1, n2 = (1 + 0.1 * rng.standard_normal((2, H))).astype(np.float32)
        layers.append(Q8DecoderLayer(q=mats["q"], k=mats["k"], v=mats["v"], o=mats["o"], gate=mats["gate"],
                                     up=mats["up"], down=mats["down"], input_norm=dev(n1), post_norm=dev(n2),
                                     eps=1e-6, bq=dev(bq), bk=dev(bk), bv=dev(bv)))
        ref_layers.append(dict(deq, bq=bq, bk=bk, bv=bv, n1=n1, n2=n2, eps=1e-6))
    emb, es = _q8(oracle, vocab, H, rng, scale=1.0)
    head, hs = _q8(oracle, vocab, H, rng, scale=0.2)
    fn = (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    model = Q8Model(layers=layers, embed=emb, lm_head=head, final_norm=dev(fn), eps=1e-6)
    ref = dict(layers=ref_layers, embed=oracle.q8_dequantize(es, vocab * H).reshape(vocab, H),
               lm_head=oracle.q8_dequantize(hs, vocab * H).reshape(vocab, H), final_norm=fn)
    return model, ref


@pytest.mark.parametrize("variant,theta,lens", [("interleaved", 1e6, [7, 30, 1]), ("split_half", 5e5, [64])])
def test_decode_step_q8_greedy_chain(oracle, variant, theta, lens):
    n_layers, hq, hkv, inter, vocab, steps = 2, 2, 1, 512, 1024, 6
    model, ref = _model(oracle, n_layers, hq, hkv, inter, vocab, seed=len(lens) * 10 + 1)
    B, D = len(lens), 128
    eng = make_engine(hq, hkv, [L + steps for L in lens], kv_dtype="f32", variant=variant, theta=theta,
                      hidden=hq * D, n_layers=n_layers, shuffle_seed=5)
    rng = np.random.default_rng(99)
    caches = []
    for l in range(n_layers):
        kc = [rng.standard_normal((L, hkv, D)).astype(np.float32) for L in lens]
        vc = [rng.standard_normal((L, hkv, D)).astype(np.float32) for L in lens]
        for b in range(B):
            eng.kv_write(l, b, torch.from_numpy(kc[b]).cuda(), torch.from_numpy(vc[b]).cuda())
        caches.append((kc, vc))
    var = oracle.ROPE_INTERLEAVED if variant == "interleaved" else oracle.ROPE_SPLIT_HALF
    cos_t, sin_t = oracle.rope_table(theta, D, max(lens) + steps)
    rl = list(lens)
    tokens = torch.from_numpy(rng.integers(0, vocab, B).astype(np.int32)).cuda()
    logits = torch.empty(B, vocab, device="cuda")
    for step in range(steps):
        tok_in = tokens.cpu().numpy()
        eng.decode_step_q8(model, list(range(B)), tokens, next_tokens=tokens, logits=logits)  # chained in place
        eng.sync()
        got, lg = tokens.cpu().numpy(), logits.cpu().numpy()
        want, ref_lg = oracle.model_decode_step(tok_in, ref["embed"], ref["layers"], ref["final_norm"],
                                                ref["lm_head"], 1e-6, caches, rl, hq, hkv, cos_t, sin_t, var)
        tol = F32_ATOL * max(1.0, np.abs(ref_lg).max())
        assert_close(lg, ref_lg, tol, what=f"logits step {step}")
        assert got.tolist() == oracle.argmax(lg).tolist(), "the pick is not the argmax of the library's logits"
        top2 = np.sort(ref_lg, axis=1)[:, -2:]
        clear = (top2[:, 1] - top2[:, 0]) > 2 * tol
        assert (got[clear] == want[clear]).all(), f"step {step}: picks {got} vs oracle {want}"
    assert [eng.seq_len(l, b) for l in range(n_layers) for b in range(B)] == [L + steps for _ in range(n_layers)
                                                                               for L in lens]
    eng.close()


def test_decode_step_q8_rejects_mismatched_models(oracle):
    from oomllama_b200 import Q8Model
    from oomllama_b200._lib import OomAttnError
    model, _ = _model(oracle, 2, 2, 1, 256, 64, seed=3)
    eng = make_engine(2, 1, [8], kv_dtype="f32", hidden=256, n_layers=1)
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    with pytest.raises(OomAttnError) as e:  # two layers, a one-layer context
        eng.decode_step_q8(model, [0], tok)
    assert e.value.code == 3
    rng = np.random.default_rng(0)
    bad = Q8Model(layers=model.layers[:1], embed=_q8(oracle, 64, 128, rng)[0], lm_head=model.lm_head,
                  final_norm=model.final_norm, eps=1e-6)
    with pytest.raises(OomAttnError) as e:  # embedding width 128, hidden 256
        eng.decode_step_q8(bad, [0], tok)
    assert e.value.code == 1
    eng.close()


def test_decode_step_q8_from_an_oom_file(oracle):
    # a 2-layer model written as an .oom file by the oracle's restatement of the converter
    # (Q8 projections, f32 norms and biases, the converter's tensor names), loaded by OomFile +
    # Q8Model.from_oom through the device repack, then greedy steps against the oracle
    from oomllama_b200 import OomFile, Q8Model
    n_layers, hq, hkv, inter, vocab, D, eps = 2, 2, 1, 512, 1024, 128, 1e-6
    H = hq * D
    rng = np.random.default_rng(21)
    w = lambda r, c, s=0.05: (rng.standard_normal((r, c)) * s).astype(np.float32)  # noqa: E731
    tensors, ref_layers = [], []
    for i in range(n_layers):
        p = f"model.layers.{i}."
        mats = {"q": w(hq * D, H), "k": w(hkv * D, H), "v": w(hkv * D, H), "o": w(H, hq * D),
                "gate": w(inter, H), "up": w(inter, H), "down": w(H, inter)}
        names = {"q": "self_attn.q_proj.weight", "k": "self_attn.k_proj.weight", "v": "self_attn.v_proj.weight",
                 "o": "self_attn.o_proj.weight", "gate": "mlp.gate_proj.weight", "up": "mlp.up_proj.weight",
                 "down": "mlp.down_proj.weight"}
        bq, bk, bv = [(rng.standard_normal(n) * 0.1).astype(np.float32) for n in (hq * D, hkv * D, hkv * D)]
        n1, n2 = (1 + 0.1 * rng.standard_normal((2, H))).astype(np.float32)
        for key, nm in names.items():
            tensors.append((p + nm, "q8", mats[key]))
        tensors += [(p + "self_attn.q_proj.bias", "f32", bq), (p + "self_attn.k_proj.bias", "f32", bk),
                    (p + "self_attn.v_proj.bias", "f32", bv), (p + "input_layernorm.weight", "f32", n1),
                    (p + "post_attention_layernorm.weight", "f32", n2)]
        deq = {k: oracle.q8_dequantize(oracle.q8_quantize(v), v.size).reshape(v.shape) for k, v in mats.items()}
        ref_layers.append(dict(deq, bq=bq, bk=bk, bv=bv, n1=n1, n2=n2, eps=eps))
    emb, head = w(vocab, H, 1.0), w(vocab, H, 0.2)
    fn = (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    tensors += [("model.embed_tokens.weight", "q8", emb), ("model.norm.weight", "f32", fn),
                ("lm_head.weight", "q8", head)]
    image = oracle.oom_image(tensors)
    lens = [9, 40]
    B, steps = len(lens), 4
    eng = make_engine(hq, hkv, [L + steps for L in lens], kv_dtype="f32", variant="interleaved", theta=1e6,
                      hidden=H, n_layers=n_layers, shuffle_seed=2)
    model = Q8Model.from_oom(OomFile(image), eng, n_layers, inter, vocab, eps)
    caches = []
    for l in range(n_layers):
        kc = [rng.standard_normal((L, hkv, D)).astype(np.float32) for L in lens]
        vc = [rng.standard_normal((L, hkv, D)).astype(np.float32) for L in lens]
        for b in range(B):
            eng.kv_write(l, b, torch.from_numpy(kc[b]).cuda(), torch.from_numpy(vc[b]).cuda())
        caches.append((kc, vc))
    cos_t, sin_t = oracle.rope_table(1e6, D, max(lens) + steps)
    ref_emb = oracle.q8_dequantize(oracle.q8_quantize(emb), emb.size).reshape(emb.shape)
    ref_head = oracle.q8_dequantize(oracle.q8_quantize(head), head.size).reshape(head.shape)
    rl = list(lens)
    tokens = torch.tensor([5, 1000], dtype=torch.int32, device="cuda")
    logits = torch.empty(B, vocab, device="cuda")
    for step in range(steps):
        tok_in = tokens.cpu().numpy()
        eng.decode_step_q8(model, list(range(B)), tokens, next_tokens=tokens, logits=logits)
        eng.sync()
        got, lg = tokens.cpu().numpy(), logits.cpu().numpy()
        want, ref_lg = oracle.model_decode_step(tok_in, ref_emb, ref_layers, fn, ref_head, eps, caches, rl, hq, hkv,
                                                cos_t, sin_t, oracle.ROPE_INTERLEAVED)
        tol = F32_ATOL * max(1.0, np.abs(ref_lg).max())
        assert_close(lg, ref_lg, tol, what=f"logits step {step}")
        top2 = np.sort(ref_lg, axis=1)[:, -2:]
        clear = (top2[:, 1] - top2[:, 0]) > 2 * tol
        assert (got[clear] == want[clear]).all()
    eng.close()


def test_prefill_step_q8_then_greedy_decode(oracle):
    # C5's order on a reduced two-layer model: a prompt of 80 tokens per sequence through the whole
    # model (tensor-core Q8 projections above 64 tokens, K-A append, K-C causal attention), the first
    # greedy pick from the last prompt token, then greedy decode steps over the bf16 cache the prefill
    # wrote.  The oracle runs the prompt token by token (one decode step per position), which is the
    # same causal computation; bf16 KV tolerance on the logits (max-abs <= 2e-3 x max(1, |logit|),
    # norm-relative <= 1e-2), picks equal wherever the oracle's top-two margin is clear.
    n_layers, hq, hkv, inter, vocab, D, n_new, steps = 2, 2, 1, 512, 1024, 128, 80, 4
    model, ref = _model(oracle, n_layers, hq, hkv, inter, vocab, seed=77)
    B = 2
    eng = make_engine(hq, hkv, [n_new + steps] * B, kv_dtype="bf16", variant="interleaved", theta=1e6,
                      hidden=hq * D, n_layers=n_layers, shuffle_seed=8)
    rng = np.random.default_rng(78)
    prompt = rng.integers(0, vocab, (B, n_new)).astype(np.int32)
    cos_t, sin_t = oracle.rope_table(1e6, D, n_new + steps)
    caches = [([np.zeros((0, hkv, D), np.float32) for _ in range(B)],
               [np.zeros((0, hkv, D), np.float32) for _ in range(B)]) for _ in range(n_layers)]
    rl = [0] * B
    for i in range(n_new):
        want, ref_lg = oracle.model_decode_step(prompt[:, i], ref["embed"], ref["layers"], ref["final_norm"],
                                                ref["lm_head"], 1e-6, caches, rl, hq, hkv, cos_t, sin_t,
                                                oracle.ROPE_INTERLEAVED, kv_bf16=True)
    logits = torch.empty(B, vocab, device="cuda")
    tokens = eng.prefill_step_q8(model, list(range(B)), torch.from_numpy(prompt).cuda(), logits=logits)
    eng.sync()
    assert [eng.seq_len(l, b) for l in range(n_layers) for b in range(B)] == [n_new] * (n_layers * B)
    for step in range(steps + 1):
        got, lg = tokens.cpu().numpy(), logits.cpu().numpy()
        tol = 2e-3 * max(1.0, np.abs(ref_lg).max())
        assert_close(lg, ref_lg, tol, 1e-2, what=f"logits after {n_new + step} tokens")
        assert got.tolist() == oracle.argmax(lg).tolist()
        top2 = np.sort(ref_lg, axis=1)[:, -2:]
        clear = (top2[:, 1] - top2[:, 0]) > 2 * tol
        assert (got[clear] == want[clear]).all(), f"picks {got} vs oracle {want}"
        if step == steps:
            break
        tok_in = got.copy()  # both follow the library's pick
        eng.decode_step_q8(model, list(range(B)), tokens, next_tokens=tokens, logits=logits)
        eng.sync()
        want, ref_lg = oracle.model_decode_step(tok_in, ref["embed"], ref["layers"], ref["final_norm"],
                                                ref["lm_head"], 1e-6, caches, rl, hq, hkv, cos_t, sin_t,
                                                oracle.ROPE_INTERLEAVED, kv_bf16=True)
    # the prefill's cache holds the oracle's rotated, bf16-rounded keys of the prompt
    k_gpu, _ = eng.kv_read(0, 1)
    kc = caches[0][0][1]  # [L, hkv, D]
    np.testing.assert_allclose(k_gpu.float().numpy()[:, :n_new], kc[:n_new].transpose(1, 0, 2), atol=0.02, rtol=0.01)
    eng.close()
