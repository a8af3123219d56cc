"""The Sticky-KV attention inside a Hugging Face Llama model.

A 2-layer ``STICKYLlamaForCausalLM`` (transformers' LlamaForCausalLM with
``STICKYLlamaAttention`` in every layer, src/models/sticky_llama_model.py:28-126),
bf16, head_dim 128 (the tensor-core decode path), run through Hugging Face's
own ``LlamaModel.forward`` with a ``DynamicCache``: Hugging Face derives the
decode positions from the cache's ``get_seq_length()`` (the true token count
of ``StickyDynamicLayer``), calls each layer's attention, and the layer's
entry presents the physical cache in the reference's order.

Every layer's attention is replayed by the oracle from the projections the
layer computed (captured with forward hooks): the prompt state, every decode
output (plain max-abs and the given-logits bound), the vote ledger, and the
window sets, Q-cache and physical K/V after each eviction cycle (bit-exact,
the oracle consuming the device's ledger, snapshotted just before each cycle).
"""

import numpy as np
import pytest
import torch

from oracle.attention import decode_attention, exact_dequant_qcache
from oracle.sticky_state import OracleStickyLayer, apply_rope, rope_cos_sin
from test_gpu_parity import output_bound

pytestmark = pytest.mark.gpu

OM, SINK, LOCAL, KW, QW = 64, 64, 128, 3, 4
PROMPT = SINK + 10 * OM


@pytest.fixture()
def sticky_model(monkeypatch):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from transformers import LlamaConfig
    import qevict_b200.kv_cache as kvmod
    from qevict_b200 import sticky_config as sc
    from qevict_b200.allocator import BudgetResult
    from qevict_b200.hf import STICKYLlamaForCausalLM
    for k, v in dict(OMEGA=OM, SINK_TOKENS=SINK, LOCAL_NUM_TOKENS=LOCAL, Q_RATIO=10, QUANTIZATION_BIT_WIDTH=8,
                     GENERATION_CONFIG={"max_new_tokens": 160}).items():
        monkeypatch.setattr(sc, k, v)
    monkeypatch.setattr(kvmod, "compute_budget", lambda **kw: BudgetResult(LOCAL, KW, QW, 0, kw.get("head_dim", 0)))
    cfg = LlamaConfig(vocab_size=1000, hidden_size=512, num_attention_heads=4, num_key_value_heads=2,
                      intermediate_size=1024, num_hidden_layers=2, max_position_embeddings=2048)
    cfg.rope_theta = 500000.0
    cfg.r_ratio, cfg.p_ratio, cfg.start_idx = 20, 50, 0
    torch.manual_seed(11)
    model = STICKYLlamaForCausalLM(cfg).to(torch.bfloat16).cuda().eval()
    return model


def test_hf_llama_decode_matches_oracle(sticky_model, monkeypatch):
    from transformers import DynamicCache
    import qevict_b200.attention as attn_mod
    from qevict_b200.layer_state import StickyLayerState
    model = sticky_model
    layers = model.model.layers
    H, G, D = 2, 2, 128
    cap = {}

    def hook(name):
        def f(mod, inp, out):
            cap[name] = out.detach().float().cpu().numpy()
        return f

    def pre_hook(name):
        def f(mod, inp):
            cap[name] = inp[0].detach().float().cpu().numpy()
        return f

    for li, layer in enumerate(layers):
        a = layer.self_attn
        a.q_proj.register_forward_hook(hook(f"q{li}"))
        a.k_proj.register_forward_hook(hook(f"k{li}"))
        a.v_proj.register_forward_hook(hook(f"v{li}"))
        a.o_proj.register_forward_pre_hook(pre_hook(f"o{li}"))
    colsums = {}
    real_prefill = attn_mod.prefill_attention

    def capture_prefill(q, k, v, colsum=True):
        out, cs = real_prefill(q, k, v, colsum)
        colsums[len(colsums)] = cs.detach().cpu().numpy()
        return out, cs
    monkeypatch.setattr(attn_mod, "prefill_attention", capture_prefill)
    # the device ledger the cycle consumes, snapshotted just before each cycle
    ledgers = {}
    real_cycle = StickyLayerState.evict_cycle

    def snap_cycle(self):
        q = self.view_q(0)
        ledgers[id(self)] = (self.view_votes(0).numpy(), None if q is None else q["scores"].numpy())
        return real_cycle(self)
    monkeypatch.setattr(StickyLayerState, "evict_cycle", snap_cycle)

    g = torch.Generator(device="cuda").manual_seed(5)
    ids = torch.randint(0, 1000, (1, PROMPT), generator=g, device="cuda")
    cache = DynamicCache()
    with torch.no_grad():
        out = model(input_ids=ids, past_key_values=cache, use_cache=True)
    cache = out.past_key_values
    assert cache.get_seq_length() == PROMPT
    cos, sin = rope_cos_sin(np.arange(PROMPT + 200), D, 500000.0, "bf16", inv_freq_dt="bf16")
    oracles, KV = [], []
    for li, layer in enumerate(layers):
        st = layer.self_attn.kv_cache.state
        q = cap[f"q{li}"][0].reshape(PROMPT, H * G, D).transpose(1, 0, 2)
        k = cap[f"k{li}"][0].reshape(PROMPT, H, D).transpose(1, 0, 2)
        v = cap[f"v{li}"][0].reshape(PROMPT, H, D).transpose(1, 0, 2)
        k = apply_rope(k, cos[:PROMPT], sin[:PROMPT], "bf16")
        o = OracleStickyLayer(H, D, OM, SINK, LOCAL, KW, QW, "bf16", 8, max_windows=st.maxW, max_context=2048,
                              window_sum="tree")
        Kr, Vr = o.prefill(k, v, colsums[li][0][:, None, :], "fp32")
        Kg, Vg = st.view_kv(0)
        np.testing.assert_array_equal(Kg.numpy(), Kr, err_msg=f"layer {li} prefill K")
        np.testing.assert_array_equal(Vg.numpy(), Vr, err_msg=f"layer {li} prefill V")
        # the cache entry Hugging Face holds is that physical cache, in the reference's order
        entry = cache.layers[li]
        assert type(entry).__name__ == "StickyDynamicLayer"
        np.testing.assert_array_equal(entry.keys[0].float().cpu().numpy(), Kr)
        assert entry.get_seq_length() == PROMPT
        oracles.append(o)
        KV.append((Kr, Vr))
    tok = out.logits[:, -1].argmax(-1, keepdim=True)
    e2e, e2e_ulp, bound_use, cycles = 0.0, 0.0, 0.0, 0
    steps = 2 * OM + 2
    for step in range(steps):
        pos = PROMPT + step
        with torch.no_grad():
            out = model(input_ids=tok, past_key_values=cache, use_cache=True)
        tok = out.logits[:, -1].argmax(-1, keepdim=True)
        assert cache.get_seq_length() == pos + 1
        for li, layer in enumerate(layers):
            st = layer.self_attn.kv_cache.state
            o = oracles[li]
            qn = apply_rope(cap[f"q{li}"][0].reshape(1, H * G, D).transpose(1, 0, 2), cos[pos:pos + 1],
                            sin[pos:pos + 1], "bf16")[:, 0]
            kn = apply_rope(cap[f"k{li}"][0].reshape(1, H, D).transpose(1, 0, 2), cos[pos:pos + 1],
                            sin[pos:pos + 1], "bf16")
            vn = cap[f"v{li}"][0].reshape(1, H, D).transpose(1, 0, 2)
            Kc = np.concatenate([KV[li][0], kn], 1)
            Vc = np.concatenate([KV[li][1], vn], 1)
            qc = None
            if o.q is not None:
                qc = {k2: o.q[k2] for k2 in ("kq", "ks", "kz", "vq", "vs", "vz")}
                qc["kdq"], qc["vdq"] = exact_dequant_qcache(o.q)
            ref, _, _ = decode_attention(qn, Kc, Vc, "bf16", qc, dequant="exact")
            got = cap[f"o{li}"][0, 0].reshape(H * G, D)
            e2e = max(e2e, float(np.abs(got - ref).max()))
            # plain max-abs beyond one bf16 ulp of the reference value: a pre-rounding
            # difference of a hair can put the two results one ulp apart (3.9e-3 at
            # |out| in [0.5, 1)); for outputs below 0.5 this is max-abs <= 2e-3 itself
            ulp = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(ref), 1e-30))) - 7)
            e2e_ulp = max(e2e_ulp, float((np.abs(got - ref) - ulp).max()))
            due = o.tokens_since + 1 == OM
            if not due:
                # the kernel's logits are only readable before the cycle rewrites the layout
                gl = st.view_logits(0).numpy()
                og, sc, qsc, ex = decode_attention(qn, Kc, Vc, "bf16", qc, dequant="exact", logits_override=gl,
                                                   return_extras=True)
                tol = output_bound(ex, "bf16", True)
                err = np.abs(got - og)
                bound_use = max(bound_use, float((err / tol).max()))
                assert (err <= tol).all(), f"layer {li} step {step}: output beyond the given-logits bound"
            else:
                _, sc, qsc = decode_attention(qn, Kc, Vc, "bf16", qc, dequant="exact")
            o.tally(Kc, sc, qsc, "bf16")
            if due:
                votes, qscores = ledgers.pop(id(st))
                o.votes[:, :Kc.shape[1]] = votes
                if qscores is not None:
                    o.q["scores"] = qscores.copy()
                Kc, Vc = o.cycle(Kc, Vc)
                ids_g, _ = st.view_sticky(0)
                np.testing.assert_array_equal(ids_g.numpy(), o.sticky_ids()[0], err_msg=f"layer {li} cycle")
                qg = st.view_q(0)
                for key in ("ids", "kq", "vq", "ks", "kz", "vs", "vz"):
                    np.testing.assert_array_equal(qg[key].numpy(), o.q[key], err_msg=f"layer {li} q.{key}")
                Kg, Vg = st.view_kv(0)
                np.testing.assert_array_equal(Kg.numpy(), Kc)
                np.testing.assert_array_equal(Vg.numpy(), Vc)
                np.testing.assert_array_equal(cache.layers[li].keys[0].float().cpu().numpy(), Kc)
                cycles += 1
            else:
                rt, at = 8e-3, 1e-6
                np.testing.assert_allclose(st.view_votes(0).numpy(), o.votes[:, :Kc.shape[1]], rtol=rt, atol=at)
            KV[li] = (Kc, Vc)
    print(f"\n[HF Llama 2 layers bf16] decode max-abs vs oracle {e2e:.3e} ({e2e_ulp:.3e} beyond one ulp of the "
          f"reference), given-logits bound use {bound_use:.3f}, cycles (all layers) {cycles}")
    assert cycles == 2 * len(layers)
    assert e2e_ulp <= 2e-3
    for layer in layers:
        assert layer.self_attn.kv_cache.state.read_error() == 0


def test_hf_generate_matches_manual_greedy(sticky_model):
    """generate() through the prepare_inputs_for_generation override (one token
    per step at the true global position, sticky_llama_model.py:72-126) gives
    the same tokens as a hand-written greedy loop over the same model."""
    from transformers import DynamicCache
    model = sticky_model
    g = torch.Generator(device="cuda").manual_seed(9)
    ids = torch.randint(0, 1000, (1, PROMPT), generator=g, device="cuda")
    n_new = OM + 6
    with torch.no_grad():
        gen = model.generate(ids, max_new_tokens=n_new, do_sample=False, past_key_values=DynamicCache(),
                             attention_mask=torch.ones_like(ids), pad_token_id=0)
    assert gen.shape[1] == PROMPT + n_new
    assert model._get_true_global_position() == PROMPT + n_new - 1
    for layer in model.model.layers:
        layer.self_attn._clean_cache()
    cache = DynamicCache()
    toks = []
    with torch.no_grad():
        out = model(input_ids=ids, past_key_values=cache, use_cache=True)
        tok = out.logits[:, -1].argmax(-1, keepdim=True)
        toks.append(tok)
        for _ in range(n_new - 1):
            out = model(input_ids=tok, past_key_values=cache, use_cache=True)
            tok = out.logits[:, -1].argmax(-1, keepdim=True)
            toks.append(tok)
    manual = torch.cat(toks, 1)
    assert torch.equal(gen[:, PROMPT:], manual), (gen[:, PROMPT:], manual)
