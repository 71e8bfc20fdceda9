"""HF integration (adakv_b200.patch) on the GPU: the registered attention
function against the oracle while the key cache grows token by token (as
HF's DynamicCache does), the batched no-mask path, and a random tiny Llama
whose full-budget sparse decode must reproduce dense decode."""
import numpy as np
import pytest
import torch

from oracle import adakv_oracle as O
from adakv_b200.synth import make_decode_case, round_to_dtype

pytestmark = pytest.mark.gpu

TOL = {"fp32": 1e-3, "bf16": 2e-2}
TORCH = {"fp32": torch.float32, "bf16": torch.bfloat16, "fp16": torch.float16}


def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


class _Layer(torch.nn.Module):
    """Stand-in for an attention module: its identity keys the centroid state;
    the dense (SDPA) branch reads the two attributes HF layers carry."""

    def __init__(self, groups=4):
        super().__init__()
        self.num_key_value_groups = groups
        self.is_causal = True


@pytest.fixture(autouse=True)
def _restore_cfg():
    from adakv_b200 import patch
    saved = dict(patch._ADAKV_CFG)
    yield
    patch._ADAKV_CFG.clear()
    patch._ADAKV_CFG.update(saved)
    patch._STATE.clear()


@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
def test_decode_steps_match_oracle_with_incremental_centroids(dtype):
    _need_cuda()
    from adakv_b200 import patch
    Hq, Hkv, D, bs, P, steps = 8, 2, 128, 16, 1000, 40
    cfg = dict(block_size=bs, avg_budget=8, k_min=2, k_max=64, n_sink_blocks=1,
               n_local_blocks=4, c_min=1, temperature=1.0)
    patch.enable_adakv(**cfg)
    case = make_decode_case(11, 1, Hq, Hkv, D, P + steps, bs, dtype)
    rng = np.random.default_rng(12)
    dt = TORCH[dtype]
    Kall = torch.from_numpy(case.K[0]).to("cuda", dt)[None]  # [1, Hkv, P+steps, D]
    Vall = torch.from_numpy(case.V[0]).to("cuda", dt)[None]
    layer = _Layer()
    scale = D ** -0.5
    # prefill pass: dense, builds the layer's centroid table
    qp = torch.from_numpy(rng.standard_normal((1, Hq, 4, D), dtype=np.float32)).to("cuda", dt)
    out_p, _ = patch.adakv_attention_forward(layer, qp, Kall[:, :, :P], Vall[:, :, :P], None, scale)
    assert out_p.shape == (1, 4, Hq, D)
    n_mismatch = 0
    for t in range(steps):
        S = P + t + 1
        # DynamicCache concatenates: a fresh tensor holding the first S tokens
        K = Kall[:, :, :S].clone()
        V = Vall[:, :, :S].clone()
        qn = rng.standard_normal((Hq, D), dtype=np.float32)
        qn = round_to_dtype(qn, dtype)
        q = torch.from_numpy(qn).to("cuda", dt)[None, :, None, :]
        out, aux = patch.adakv_attention_forward(layer, q, K, V, None, scale)
        assert aux is None and out.shape == (1, 1, Hq, D) and out.dtype == dt
        ref = O.decode_step(qn, case.K[0][:, :S], case.V[0][:, :S], block_size=bs,
                            avg_budget=8, k_min=2, k_max=64, sm_scale=scale)
        err = np.abs(out[0, 0].float().cpu().numpy() - ref["out"]).max()
        if err >= TOL[dtype]:
            n_mismatch += 1
    # every step within tolerance (a selection near-tie could move one step)
    assert n_mismatch == 0
    st = patch._STATE[id(layer)]
    assert st.n == P + steps
    # the incrementally maintained table equals a rebuild from all keys
    nb = (P + steps + bs - 1) // bs
    full = O.build_centroids(case.K[0][:, : P + steps], bs)
    got = st.cbuf[0, :, :nb].cpu().numpy()
    assert np.array_equal(got, full)


def test_batched_no_mask_matches_per_sequence():
    _need_cuda()
    from adakv_b200 import patch
    Hq, Hkv, D, bs, S, B = 8, 2, 64, 16, 777, 3
    patch.enable_adakv(block_size=bs, avg_budget=6, k_max=64)
    case = make_decode_case(21, B, Hq, Hkv, D, S, bs, "bf16")
    dt = torch.bfloat16
    K = torch.from_numpy(case.K).to("cuda", dt)
    V = torch.from_numpy(case.V).to("cuda", dt)
    q = torch.from_numpy(case.q).to("cuda", dt)[:, :, None, :]
    out, _ = patch.adakv_attention_forward(_Layer(), q, K, V, None, D ** -0.5)
    assert out.shape == (B, 1, Hq, D)
    for b in range(B):
        ref = O.decode_step(case.q[b], case.K[b], case.V[b], block_size=bs, avg_budget=6,
                            k_max=64, sm_scale=D ** -0.5)
        err = np.abs(out[b, 0].float().cpu().numpy() - ref["out"]).max()
        assert err < TOL["bf16"], f"sequence {b}: {err:.3e}"


def test_disabled_and_masked_batches_go_dense():
    _need_cuda()
    from adakv_b200 import patch
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    sdpa = ALL_ATTENTION_FUNCTIONS["sdpa"]
    Hq, Hkv, D, S = 8, 2, 64, 300
    g = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randn((2, Hq, 1, D), device="cuda", generator=g)
    K = torch.randn((2, Hkv, S, D), device="cuda", generator=g)
    V = torch.randn((2, Hkv, S, D), device="cuda", generator=g)
    layer = _Layer(Hq // Hkv).eval()
    mask = torch.ones((2, 1, 1, S), dtype=torch.bool, device="cuda")
    mask[1, :, :, :10] = False  # left padding on the second sequence
    ref, _ = sdpa(layer, q, K, V, attention_mask=mask, scaling=D ** -0.5)
    out, _ = patch.adakv_attention_forward(layer, q, K, V, mask, D ** -0.5)
    assert torch.equal(out, ref)
    patch.disable_adakv()
    ref1, _ = sdpa(layer, q[:1], K[:1], V[:1], attention_mask=None, scaling=D ** -0.5)
    out1, _ = patch.adakv_attention_forward(layer, q[:1], K[:1], V[:1], None, D ** -0.5)
    assert torch.equal(out1, ref1)


@pytest.mark.parametrize("sel", ["h2o", "snapkv"])
def test_eviction_baselines_through_patch_match_oracle(sel):
    """selection="h2o" / "snapkv": the prefill call freezes each head's retained
    blocks (the oracle's mask), and the decode steps attend to the frozen set
    plus the sink and the current local window (the oracle's frozen attention)."""
    _need_cuda()
    from adakv_b200 import patch
    from adakv_b200.synth import make_prefill_case
    Hq, Hkv, D, bs, P, steps = 8, 2, 64, 16, 700, 20
    cfg = dict(block_size=bs, avg_budget=12, n_sink_blocks=1, n_local_blocks=3, c_min=1,
               selection=sel, obs_window=32, pool_kernel=7)
    patch.enable_adakv(**cfg)
    Q, K, V, _ = make_prefill_case(40, Hq, Hkv, D, P + steps)
    Kt = torch.from_numpy(K).cuda()[None]
    Vt = torch.from_numpy(V).cuda()[None]
    layer = _Layer()
    out_p, _ = patch.adakv_attention_forward(layer, torch.from_numpy(Q[:, :P]).cuda()[None],
                                             Kt[:, :, :P], Vt[:, :, :P], None, D ** -0.5)
    g = Hq // Hkv
    Kq = np.repeat(K[:, :P], g, axis=0)
    imp = (O.h2o_key_importance(Q[:, :P], Kq) if sel == "h2o"
           else O.snapkv_key_importance(Q[:, :P], Kq, 32, 7))
    fmask = O.retain_blocks(imp, bs, P, 12, 1, 3, 1)
    assert np.array_equal(patch._FROZEN[id(layer)].cpu().numpy(), fmask)
    rng = np.random.default_rng(41)
    for t in range(steps):
        S = P + t + 1
        qn = rng.standard_normal((Hq, D)).astype(np.float32)
        q = torch.from_numpy(qn).cuda()[None, :, None, :]
        out, _ = patch.adakv_attention_forward(layer, q, Kt[:, :, :S], Vt[:, :, :S], None, D ** -0.5)
        dm = O.frozen_decode_mask(fmask, (S + bs - 1) // bs, 1, 3)
        ref = O.attend_mask(qn, K[:, :S], V[:, :S], dm, bs)
        assert np.abs(out[0, 0].cpu().numpy() - ref).max() < TOL["fp32"]


@pytest.mark.parametrize("dtype,Hq,Hkv,D,S", [("fp32", 6, 6, 64, 384), ("fp32", 8, 2, 128, 517),
                                               ("bf16", 16, 4, 128, 1500), ("fp16", 8, 2, 64, 300)])
def test_key_importance_matches_oracle(dtype, Hq, Hkv, D, S):
    """adakv_key_importance (GQA, per KV head) against the float64 oracle at the
    reference's own bar (1e-4 relative), and the retained masks equal."""
    _need_cuda()
    from adakv_b200 import baselines_rt as RT
    from adakv_b200.synth import make_prefill_case
    Q, K, _, _ = make_prefill_case(42, Hq, Hkv, D, S)
    Q, K = round_to_dtype(Q, dtype), round_to_dtype(K, dtype)
    dt = TORCH[dtype]
    q = torch.from_numpy(Q).cuda().to(dt)[None]
    k = torch.from_numpy(K).cuda().to(dt)[None]
    Kq = np.repeat(K, Hq // Hkv, axis=0)
    for n_query, ref in ((S, O.h2o_key_importance(Q, Kq)),
                         (32, O.snapkv_key_importance(Q, Kq, 32, 1))):
        got = RT.key_importance(q, k, n_query).cpu().numpy()
        rel = np.abs(got - ref).max() / np.abs(ref).max()
        assert rel < 1e-4, f"n_query {n_query}: rel err {rel:.2e}"
    # the reference-layout entry points (keys expanded) and the retained masks
    if Hq == Hkv:
        Qt, Kt = torch.from_numpy(Q).cuda(), torch.from_numpy(K).cuda()
        for budget in (6, 8, 12):
            m = RT.h2o_retained_mask_torch(Qt, Kt, 16, budget, 1, 2, 1).cpu().numpy()
            assert np.array_equal(m, O.retain_blocks(O.h2o_key_importance(Q, K), 16, S, budget, 1, 2, 1))
            m = RT.snapkv_retained_mask_torch(Qt, Kt, 16, budget, 32, 7, 1, 2, 1).cpu().numpy()
            ref = O.retain_blocks(O.snapkv_key_importance(Q, K, 32, 7), 16, S, budget, 1, 2, 1)
            assert np.array_equal(m, ref)


def _tiny_llama(dtype):
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(0)
    cfg = LlamaConfig(hidden_size=512, intermediate_size=1024, num_attention_heads=8,
                      num_key_value_heads=2, num_hidden_layers=2, vocab_size=512,
                      max_position_embeddings=4096, pad_token_id=0, eos_token_id=1,
                      bos_token_id=2)
    return LlamaForCausalLM(cfg).to("cuda", dtype).eval()


def test_patch_model_full_budget_generate_equals_dense():
    """With every block selected, sparse decode is dense decode: greedy tokens
    agree and the decode logits agree to fp32 accumulation noise."""
    _need_cuda()
    from adakv_b200 import patch
    model = _tiny_llama(torch.float32)
    ids = torch.randint(3, 512, (1, 700), device="cuda", generator=torch.Generator(
        device="cuda").manual_seed(1))
    n_new = 12
    with torch.no_grad():
        dense = model.generate(ids, max_new_tokens=n_new, do_sample=False,
                               output_logits=True, return_dict_in_generate=True)
        patch.patch_model(model, block_size=16, avg_budget=4096, k_min=4096, k_max=4096)
        sparse = model.generate(ids, max_new_tokens=n_new, do_sample=False,
                                output_logits=True, return_dict_in_generate=True)
    assert torch.equal(dense.sequences, sparse.sequences)
    for a, b in zip(dense.logits[1:], sparse.logits[1:]):
        assert (a - b).abs().max().item() < 1e-3
    assert len(patch._STATE) == 2  # one centroid table per layer


def test_patch_model_sparse_generate_runs_bf16():
    _need_cuda()
    from adakv_b200 import patch
    from adakv_b200 import attention as A
    model = _tiny_llama(torch.bfloat16)
    ids = torch.randint(3, 512, (1, 1500), device="cuda", generator=torch.Generator(
        device="cuda").manual_seed(2))
    patch.patch_model(model, block_size=16, avg_budget=16, k_max=64)
    A.reset_budget_trace()
    with torch.no_grad():
        out = model.generate(ids, max_new_tokens=8, do_sample=False, output_logits=True,
                             return_dict_in_generate=True)
    trace = A.get_budget_trace()
    A.stop_budget_trace()
    assert out.sequences.shape == (1, 1508)
    assert all(torch.isfinite(l).all() for l in out.logits)
    # 2 layers x 7 decode calls recorded, mean budget near the target of 16
    assert len(trace) == 14
    assert all(8 <= t <= 64 for t in trace)


def test_minmax_estimator_through_patch():
    _need_cuda()
    from adakv_b200 import patch
    Hq, Hkv, D, bs, P, steps = 8, 2, 64, 16, 700, 5
    patch.enable_adakv(block_size=bs, avg_budget=8, k_max=64, estimator="minmax")
    case = make_decode_case(14, 1, Hq, Hkv, D, P + steps, bs, "fp32")
    Kall = torch.from_numpy(case.K[0]).cuda()[None]
    Vall = torch.from_numpy(case.V[0]).cuda()[None]
    layer = _Layer()
    rng = np.random.default_rng(15)
    qp = torch.from_numpy(rng.standard_normal((1, Hq, 3, D), dtype=np.float32)).cuda()
    patch.adakv_attention_forward(layer, qp, Kall[:, :, :P], Vall[:, :, :P], None, D ** -0.5)
    for t in range(steps):
        S = P + t + 1
        qn = rng.standard_normal((Hq, D), dtype=np.float32)
        q = torch.from_numpy(qn).cuda()[None, :, None, :]
        out, _ = patch.adakv_attention_forward(layer, q, Kall[:, :, :S].clone(),
                                               Vall[:, :, :S].clone(), None, D ** -0.5)
        ref = O.decode_step(qn, case.K[0][:, :S], case.V[0][:, :S], block_size=bs, avg_budget=8,
                            k_max=64, sm_scale=D ** -0.5, estimator="minmax")
        err = np.abs(out[0, 0].cpu().numpy() - ref["out"]).max()
        assert err < TOL["fp32"], f"step {t}: {err:.3e}"


def test_static_cache_generate_matches_dynamic_cache():
    """adakv_b200.hf_cache.AdaKVStaticCache: preallocated per-layer K/V whose
    update writes the tokens and rebuilds the touched blocks' centroids in one
    launch (the prompt's table while the prefill writes the cache).  Greedy
    generation through it equals generation through HF's DynamicCache, and
    every layer's table equals a fresh build from the cache's keys."""
    _need_cuda()
    from adakv_b200 import _lib, patch
    from adakv_b200.hf_cache import AdaKVStaticCache
    model = _tiny_llama(torch.float32)
    ids = torch.randint(3, 512, (2, 900), device="cuda", generator=torch.Generator(
        device="cuda").manual_seed(3))
    n_new = 10
    patch.patch_model(model, block_size=16, avg_budget=8, k_max=64)
    with torch.no_grad():
        dyn = model.generate(ids, max_new_tokens=n_new, do_sample=False, output_logits=True,
                             return_dict_in_generate=True)
        cache = AdaKVStaticCache(model.config, max_cache_len=ids.shape[1] + n_new)
        sta = model.generate(ids, past_key_values=cache, max_new_tokens=n_new, do_sample=False,
                             output_logits=True, return_dict_in_generate=True)
    assert torch.equal(dyn.sequences, sta.sequences)
    for a, b in zip(dyn.logits, sta.logits):
        assert (a - b).abs().max().item() < 1e-3
    S = ids.shape[1] + n_new - 1  # the last generated token is never fed back
    L = _lib.lib()
    for layer in cache.layers:
        assert layer.fused and layer.get_seq_length() == S
        B, Hkv, _, D = layer.keys.shape
        ref = torch.empty_like(layer.centroid)
        geo = _lib.geometry(B, Hkv, Hkv, D, 16, S, ref.shape[2], _lib.TORCH_DTYPES[torch.float32])
        _lib.check(L.adakv_centroid_build(geo, _lib.view4(layer.keys), None, ref.data_ptr(),
                                          _lib.stream_ptr(ref.device)))
        nb = -(-S // 16)
        assert torch.equal(layer.centroid[:, :, :nb], ref[:, :, :nb])
    with pytest.raises(ValueError, match="holds"):
        cache.layers[0].update(torch.zeros(2, 2, 2, 64, device="cuda"),
                               torch.zeros(2, 2, 2, 64, device="cuda"))


def test_key_importance_batched_rows_are_independent():
    """B = 2 in one launch: each sequence's importance equals its own oracle."""
    _need_cuda()
    from adakv_b200 import baselines_rt as RT
    from adakv_b200.synth import make_prefill_case
    Hq, Hkv, D, S = 8, 2, 128, 333
    cases = [make_prefill_case(50 + b, Hq, Hkv, D, S) for b in range(2)]
    q = torch.stack([torch.from_numpy(c[0]) for c in cases]).cuda()
    k = torch.stack([torch.from_numpy(c[1]) for c in cases]).cuda()
    got = RT.key_importance(q, k, S).cpu().numpy().reshape(2, Hq, S)
    for b, (Q, K, _, _) in enumerate(cases):
        ref = O.h2o_key_importance(Q, np.repeat(K, Hq // Hkv, axis=0))
        assert np.abs(got[b] - ref).max() / np.abs(ref).max() < 1e-4
