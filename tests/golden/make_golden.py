"""Generate golden vectors by running the reference's own code on CPU.

Run once in a container that has the reference source tree (it is read-only
and not present on the GPU host):

    HOME_SEEK_REF=/path/to/home-seek/src python tests/golden/make_golden.py

Every input is regenerated from the seeds in oracle/inputs.py; the fixtures
store the reference outputs (and the small inputs, for convenience) in
tests/golden/*.npz. Reference entry points exercised:
  home_seek.router.compute_expert_affinity_with_bias        (router.py:22-36)
  HomeSeekInferenceEngine._compute_hash_experts              (engine.py:1018-1023)
  home_seek.fused_moe.FusedMoEFFN.forward                    (fused_moe.py:447-551)
  home_seek.fused_moe.SharedExpertFFN.forward + load_fp8_weight
                                                             (fused_moe.py:573-598,
                                                              weight_loader.py:22-32)
  HomeSeekInferenceEngine._mtp_verify_batched (greedy loop)  (engine.py:2431-2540)
  tests/_reference.py expand_to_fused / reduce_fused          (_reference.py:52-121)
  the MTP decode loop (gen_mtp): generate()'s greedy loop body (engine.py:
  2809-2922, restated in the harness) around the reference's own
  _forward_layer / _forward_ffn (engine.py:2653-2688, 1413-1541),
  _mtp_generate_draft / _mtp_forward_draft / _mtp_finalize (engine.py:
  2036-2133, 2251-2338) and _mtp_verify_batched (engine.py:2431-2540)
"""
from __future__ import annotations

import os
import sys
from pathlib import Path
from unittest.mock import MagicMock

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from oracle import inputs as I  # noqa: E402
from oracle import moe as O  # noqa: E402


def _ref_path() -> Path:
    p = os.environ.get("HOME_SEEK_REF")
    if p:
        return Path(p)
    raise SystemExit("set HOME_SEEK_REF to the reference's src directory")


def _bf16_np(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _fp4_loader_ref(load):
    """Wrap the oracle's seeded uint8 arrays in the reference's 6-tuple format:
    int8 packed data and float8_e8m0fnu scales (what _make_raw_entry keeps)."""
    def fn(layer, eid):
        w1, s1, w3, s3, w2, s2 = load(int(eid))
        c = lambda a: torch.from_numpy(a).view(torch.int8)  # noqa: E731
        s = lambda a: torch.from_numpy(a).view(torch.float8_e8m0fnu)  # noqa: E731
        return (c(w1), s(s1), c(w3), s(s3), c(w2), s(s2))
    return fn


def gen_router(out):
    from home_seek.router import compute_expert_affinity_with_bias
    cases = {
        "small": (I.hidden(5, 512, seed=10), *I.router_weights(16, 512, seed=11)),
        "cfg0": (I.hidden(3, 4096, seed=0), *I.router_weights(256, 4096, seed=1)),
        "t24": (I.hidden(24, 4096, seed=12), *I.router_weights(256, 4096, seed=13)),
    }
    h, gate, bias = I.hidden(4, 512, seed=14), *I.router_weights(32, 512, seed=15)
    gate = gate.clone()
    gate[9] = gate[5]  # identical rows -> identical logits: stable order must pick 5 before 9
    gate[20] = gate[5]
    bias = bias.clone()
    bias[9] = bias[5]
    bias[20] = bias[5]
    cases["ties"] = (h, gate, bias)
    for name, (h, gate, bias) in cases.items():
        idx, w = compute_expert_affinity_with_bias(h, gate, bias, top_k=6, routed_scaling_factor=1.5)
        logits = torch.matmul(h, gate.t()) + bias
        out[f"router_{name}_idx"] = idx.numpy()
        out[f"router_{name}_w"] = w.numpy()
        out[f"router_{name}_logits"] = _bf16_np(logits)


def gen_hash(out):
    from home_seek.inference_engine import HomeSeekInferenceEngine
    from home_seek.model_config import DeepSeekV4FlashConfig
    eng = HomeSeekInferenceEngine.__new__(HomeSeekInferenceEngine)
    eng.config = DeepSeekV4FlashConfig(num_experts_per_tok=6, num_hash_layers=3)
    tid = I.tid2eid(1000, 256, 6, seed=3)
    ids = torch.tensor([[5, 10, 15, 999, 0]], dtype=torch.int64)
    eids, w = eng._compute_hash_experts(ids, 0, tid)
    out["hash_ids"] = ids.numpy()
    out["hash_eids"] = eids.numpy()
    out["hash_w"] = w.numpy()


def gen_moe(out):
    from home_seek.fused_moe import FusedMoEFFN, SharedExpertFFN
    from home_seek.inference_engine.weight_loader import load_fp8_weight
    from home_seek.router import compute_expert_affinity_with_bias

    def run(shape, T, seed, name, hash_route=False):
        h = I.hidden(T, shape.D, seed=seed)
        if hash_route:
            tid = I.tid2eid(97, shape.E, shape.K, seed=seed + 1)
            ids = torch.arange(T, dtype=torch.int64) * 7 % 97
            idx = tid[ids]
            w = torch.full((T, shape.K), 1.0 / shape.K)
        else:
            gate, bias = I.router_weights(shape.E, shape.D, seed=seed + 1)
            idx, w = compute_expert_affinity_with_bias(h, gate, bias, top_k=shape.K, routed_scaling_factor=1.5)
        load = I.make_loader(shape)
        ffn = FusedMoEFFN(num_experts=shape.E, intermediate_size=shape.I, hidden_size=shape.D)
        assert not ffn.use_triton  # CPU: the _forward_legacy cuBLAS-branch math on ATen
        routed = ffn.forward(h, idx, w, _fp4_loader_ref(load), 5)
        w13, s13, w2, s2 = I.shared_fp8(shape.D, shape.I_sh, seed=seed + 2)
        t8 = lambda a: torch.from_numpy(np.ascontiguousarray(a)).view(torch.float8_e4m3fn)  # noqa: E731
        u8 = lambda a: torch.from_numpy(np.ascontiguousarray(a))  # noqa: E731
        sw1 = load_fp8_weight(t8(w13[0]), u8(s13[0]))
        sw3 = load_fp8_weight(t8(w13[1]), u8(s13[1]))
        sw2 = load_fp8_weight(t8(w2), u8(s2))
        sh = SharedExpertFFN(hidden_size=shape.D, intermediate_size=shape.I_sh)
        shared = sh.forward(h.unsqueeze(0), sw1, sw3, sw2, h.dtype)[0]
        full = routed + shared
        out[f"moe_{name}_idx"] = idx.numpy()
        out[f"moe_{name}_w"] = w.numpy()
        out[f"moe_{name}_routed"] = _bf16_np(routed)
        out[f"moe_{name}_out"] = _bf16_np(full)
        out[f"moe_{name}_meta"] = np.array([shape.D, shape.I, shape.E, shape.I_sh, shape.K, T, seed], dtype=np.int64)

    for T in (1, 3, 5, 24):
        run(I.SMALL, T, 20 + T, f"small_t{T}")
    run(I.SMALL, 6, 40, "small_hash", hash_route=True)
    run(I.CONFIG0, 3, 0, "cfg0")


def gen_accept(out):
    """Greedy acceptance through the reference's _mtp_verify_batched, with a
    mocked forward whose output becomes the logits exactly (identity lm_head,
    hc_mult=1, no norm, no hc head)."""
    from home_seek.inference_engine import HomeSeekInferenceEngine
    V = 256

    def verify(logits_rows: torch.Tensor, ids: list[int]):
        eng = HomeSeekInferenceEngine.__new__(HomeSeekInferenceEngine)
        eng._log = lambda m: None
        eng.config = MagicMock()
        eng.config.num_hidden_layers = 1
        eng.config.hc_mult = 1
        eng.layer_states = {}
        eng._compressors = {}
        eng._global_pos = 0
        eng.embed = torch.zeros(V, V, dtype=torch.bfloat16)
        eng.lm_head = torch.eye(V, dtype=torch.bfloat16)
        eng.norm_weight = None
        eng.hc_head_fn = None
        eng._get_layer_weights = lambda i: {}
        eng._forward_layer = lambda h, lw, i, ids_: (logits_rows.view(1, -1, 1, V).to(torch.bfloat16), set())
        main = torch.tensor([[ids[0]]], dtype=torch.int64)
        drafts = torch.tensor([ids[1:]], dtype=torch.int64)
        n, bonus = eng._mtp_verify_batched(drafts, 0.0, main_pred_id=main)
        return n, int(bonus.argmax(dim=-1).item())

    g = torch.Generator().manual_seed(5)
    rows, ids_all, n_all, nxt_all = [], [], [], []
    for case in range(12):
        lg = (torch.randn(3, V, generator=g) * 3).to(torch.bfloat16)
        am = lg.float().argmax(dim=-1).tolist()
        # case % 4: 0 -> reject first, 1 -> accept one, 2 -> accept both, 3 -> tie at argmax
        ids = [7, (am[0] + 1) % V, 11]
        if case % 4 >= 1:
            ids[1] = am[0]
        if case % 4 == 2:
            ids[2] = am[1]
        if case % 4 == 3:
            j = (am[0] + 17) % V
            lg[0, j] = lg[0, am[0]]  # duplicate max later in the row... or earlier
            lg[0, (am[0] + V - 3) % V] = lg[0, am[0]]
            ids[1] = int(lg[0].float().argmax())
        n, nxt = verify(lg, ids)
        rows.append(lg)
        ids_all.append(ids)
        n_all.append(n)
        nxt_all.append(nxt)
    out["accept_logits"] = _bf16_np(torch.stack(rows))
    out["accept_ids"] = np.array(ids_all, dtype=np.int64)
    out["accept_n"] = np.array(n_all, dtype=np.int32)
    out["accept_next"] = np.array(nxt_all, dtype=np.int64)


def gen_permute(out):
    import importlib.util
    spec = importlib.util.spec_from_file_location("_hs_ref_tests", _ref_path().parent / "tests" / "_reference.py")
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    # The reference compiles elementwise_fma with Inductor, whose CPU build uses
    # -ffp-contract=off: a separate multiply and add. Run the same arithmetic
    # eagerly (Inductor's C++ toolchain is not available here).
    ref.elementwise_fma = lambda a, b, c: a * b + c
    g = torch.Generator().manual_seed(9)
    T, K, E, D = 7, 4, 8, 64
    idx = torch.randint(-1, E, (T, K), generator=g)
    idx[2, 1] = idx[2, 0]  # a duplicate expert in one row
    x = torch.randn(T, D, generator=g).to(torch.bfloat16)
    w = torch.rand(T, K, generator=g)
    pos, p2e, cnt, n = O.permute_plan(idx.numpy(), E)
    xe = ref.expand_to_fused(x, torch.from_numpy(pos).long(), torch.from_numpy(p2e[: T * K]).long())
    red = ref.reduce_fused(xe, w, torch.from_numpy(pos).long())
    out["perm_idx"] = idx.numpy()
    out["perm_x"] = _bf16_np(x)
    out["perm_w"] = w.numpy()
    out["perm_pos"] = pos
    out["perm_xe"] = _bf16_np(xe)
    out["perm_reduced"] = _bf16_np(red)


def _mtp_engine(shape, model):
    """A reference engine object (no __init__: that loads a checkpoint and
    touches CUDA) whose own layer, FFN, draft and verify code runs on the small
    seeded model, with attention off (hc_mult = 1, no MHC weights, the
    attention blocks return zeros) and the weight stores replaced by the
    seeded tensors in the formats the reference's loaders return."""
    from collections import OrderedDict

    from home_seek.fused_moe import FusedMoEFFN, SharedExpertFFN
    from home_seek.inference_engine import HomeSeekInferenceEngine
    from home_seek.inference_engine.weight_loader import load_fp8_weight
    from home_seek.model_config import DeepSeekV4FlashConfig
    s = shape
    eng = HomeSeekInferenceEngine.__new__(HomeSeekInferenceEngine)
    eng._log = lambda m: None
    eng.verbose = False
    eng.config = DeepSeekV4FlashConfig(num_hidden_layers=s.L, hidden_size=s.D, moe_intermediate_size=s.I,
                                       vocab_size=s.V, n_routed_experts=s.E, num_experts_per_tok=s.K,
                                       num_hash_layers=s.hash_layers, shared_expert_intermediate_size=s.I_sh,
                                       hc_mult=1)
    eng.device = torch.device("cpu")
    eng._is_multigpu = False
    eng._hot_expert_set = set()
    eng._hot_expert_set_by_layer = {}
    eng._deq_cache = OrderedDict()
    eng._fused_moe = FusedMoEFFN(num_experts=s.E, intermediate_size=s.I, hidden_size=s.D)
    assert not eng._fused_moe.use_triton  # CPU: _forward_legacy
    eng._shared_ffn = SharedExpertFFN(hidden_size=s.D, intermediate_size=s.I_sh)
    eng.layer_states = {}
    eng._compressors = {}
    eng._global_pos = 0
    eng.embed = model["embed"]
    eng.lm_head = model["lm_head"]
    eng.norm_weight = model["norm_w"]
    eng.hc_head_fn = None
    eng._mtp_weights = {"mtp.0.e_proj.weight": model["e_proj"], "mtp.0.h_proj.weight": model["h_proj"],
                        "mtp.0.enorm.weight": model["enorm_w"], "mtp.0.hnorm.weight": model["hnorm_w"],
                        "mtp.0.norm.weight": model["mtp_norm_w"], "mtp.0.ffn_norm.weight": model["ln_w"][s.L],
                        "mtp.0.ffn.gate.weight": model["gate"][s.L], "mtp.0.ffn.gate.bias": model["bias"][s.L]}
    zeros_like_rows = lambda h, *a, **k: torch.zeros_like(h)  # noqa: E731  (attention off)
    eng._forward_attn = zeros_like_rows
    eng._mtp_attn_1tok = zeros_like_rows

    def layer_weights(i):
        lw = {"ffn_norm.weight": model["ln_w"][i], "ffn.gate.weight": model["gate"][i],
              "ffn.gate.bias": model["bias"][i]}
        if i in model["tid2eid"]:
            lw["ffn.gate.tid2eid"] = model["tid2eid"][i]
        return lw
    eng._get_layer_weights = layer_weights
    fp4 = [_fp4_loader_ref(model["experts"][l]) for l in range(s.L + 1)]
    # the routed experts of layer l as FusedMoEFFN's loader receives them (the
    # FP4 6-tuple; it replaces _load_bf16_deq, whose cache key omits the layer)
    eng._load_bf16_deq = lambda layer, eid: fp4[layer](layer, eid)

    def shared(layer):  # what _get_shared_expert returns for a cached FP8 entry
        w13, s13, w2, s2 = model["shared"][layer]
        t8 = lambda a: torch.from_numpy(np.ascontiguousarray(a)).view(torch.float8_e4m3fn)  # noqa: E731
        u8 = lambda a: torch.from_numpy(np.ascontiguousarray(a))  # noqa: E731
        return (load_fp8_weight(t8(w13[0]), u8(s13[0])), load_fp8_weight(t8(w13[1]), u8(s13[1])),
                load_fp8_weight(t8(w2), u8(s2)))
    eng._get_shared_expert = shared

    def mtp_expert(eid):  # _mtp_load_expert's entry: (data, f32 scale, "fp4") triples
        w1, s1, w3, s3, w2, s2 = fp4[s.L](s.L, eid)
        return tuple((w, sc.to(torch.float32), "fp4") for w, sc in ((w1, s1), (w3, s3), (w2, s2)))
    eng._mtp_load_expert = mtp_expert
    return eng


def gen_mtp(out, iterations: int = 16, first_token: int = 100):
    """The greedy MTP decode loop of generate() (engine.py:2809-2922, t = 0,
    mtp_num_draft = M, no stop token) on the small seeded model: main T = 1
    step, _mtp_generate_draft, _mtp_verify_batched, and the loop's
    bookkeeping. Records the token stream, every decision's inputs and
    outcome, and every logits row an argmax was taken of."""
    from home_seek.utils import rms_norm
    s = I.MTP_SMALL
    model = I.mtp_model(s)
    eng = _mtp_engine(s, model)
    eps = eng.config.rms_norm_eps
    next_id = torch.tensor([[first_token]], dtype=torch.int64)
    generated = []
    recs, lg_main, lg_draft, lg_verify = [], [], [], []
    for _ in range(iterations):
        # main step (engine.py:2811-2853)
        h = eng.embed[next_id].to(torch.bfloat16)
        h = h.unsqueeze(2).expand(-1, -1, eng.config.hc_mult, -1)
        for layer_idx in range(s.L):
            h, _ = eng._forward_layer(h, eng._get_layer_weights(layer_idx), layer_idx, next_id)
        last_h = h
        h_3d = rms_norm(h.sum(dim=2), eng.norm_weight, eps)
        logits = torch.matmul(h_3d.to(eng.lm_head.dtype), eng.lm_head.t())
        main_in = int(next_id)
        next_id = logits[:, -1].argmax(dim=-1, keepdim=True)
        generated.append(int(next_id))
        lg_main.append(logits[0, -1])
        # draft (engine.py:2867-2870); the logits rows of its argmaxes are
        # captured at the head matmul (kept for the parity tests' margins)
        heads = []
        draft_ids, n_draft = _draft_with_logits(eng, last_h, s.M, next_id, heads)
        assert n_draft == s.M
        # verify (engine.py:2885-2886)
        n_acc, bonus_logits = _verify_with_logits(eng, draft_ids, next_id, lg_verify)
        d = [int(v) for v in draft_ids[0]]
        rec = [main_in, int(next_id), d[0], d[1], n_acc]
        if n_acc > 0:  # engine.py:2893-2916
            generated.extend(d[:n_acc])
            next_id = bonus_logits.argmax(dim=-1, keepdim=True)
            generated.append(int(next_id))
        rec.append(int(next_id))
        recs.append(rec)
        lg_draft.append(torch.stack(heads))
    out["mtp_tokens"] = np.array(generated, dtype=np.int64)
    out["mtp_records"] = np.array(recs, dtype=np.int64)  # main_in, main_pred, d1, d2, n_acc, next_id
    out["mtp_logits_main"] = _bf16_np(torch.stack(lg_main))
    out["mtp_logits_draft"] = _bf16_np(torch.stack(lg_draft))
    out["mtp_logits_verify"] = _bf16_np(torch.stack(lg_verify))
    out["mtp_meta"] = np.array([s.D, s.I, s.E, s.I_sh, s.K, s.V, s.L, s.hash_layers, s.M, iterations,
                                first_token], dtype=np.int64)


def _draft_with_logits(eng, last_h, M, next_id, rows):
    """eng._mtp_generate_draft(last_h, M, 0.0, last_token_id=next_id), with the
    logits of each draft step captured at its matmul with the head."""
    real = eng.lm_head

    class _Capture:
        dtype = real.dtype

        def t(self):
            return _CaptureT()

    class _CaptureT:
        def __rmatmul__(self, x):
            lg = x @ real.t()
            rows.append(lg[0, -1])
            return lg
    eng.lm_head = _Capture()
    try:
        return eng._mtp_generate_draft(last_h, M, 0.0, last_token_id=next_id)
    finally:
        eng.lm_head = real


def _verify_with_logits(eng, draft_ids, main_pred, rows):
    """eng._mtp_verify_batched(draft_ids, 0.0, main_pred_id=main_pred), with
    the [T, V] logits of its fused forward captured at torch.matmul."""
    real_matmul = torch.matmul
    seen = []

    def hook(a, b, *args, **kw):
        r = real_matmul(a, b, *args, **kw)
        if r.dim() == 3 and r.shape[-1] == eng.lm_head.shape[0]:
            seen.append(r[0])
        return r
    torch.matmul = hook
    try:
        n, bonus = eng._mtp_verify_batched(draft_ids, 0.0, main_pred_id=main_pred)
    finally:
        torch.matmul = real_matmul
    assert len(seen) == 1
    rows.append(seen[0])
    return n, bonus


def gen_verify_state(out):
    """The state handling of the reference's _mtp_verify_batched (engine.py:
    2443-2459, 2500-2538) on seeded layer states: a mocked forward appends KV
    rows, a compressed row and rewrites the compressor (oracle/verify_state.py
    forward_mutation), its logits rows are chosen so n_accept is 0, 1 or 2 of
    T = 3 positions; the states and position after the call are recorded."""
    from types import SimpleNamespace

    from home_seek.inference_engine import HomeSeekInferenceEngine
    from home_seek.inference_engine.layer_state import LayerState
    from oracle import verify_state as VS
    V = 64
    for case, n_want in enumerate((0, 1, 2)):
        before = VS.scenario_states(seed=7 + case)
        eng = HomeSeekInferenceEngine.__new__(HomeSeekInferenceEngine)
        eng._log = lambda m: None
        eng.config = MagicMock()
        eng.config.num_hidden_layers = len(before)
        eng.config.hc_mult = 1
        eng.config.rms_norm_eps = 1e-6
        eng.layer_states, eng._compressors = {}, {}
        for l, st in before.items():
            ls = LayerState(device="cpu")
            ls.kv_latent_cache = st["kv"].clone()
            ls.compressed_kv_data = st["cdata"].clone()
            ls.compressed_kv_idx = st["cidx"].clone()
            eng.layer_states[l] = ls
            acc, kvs, scs = st["comp"]
            eng._compressors[l] = SimpleNamespace(accumulated=acc, kv_state=kvs.clone(), score_state=scs.clone())
        eng._global_pos = 40
        eng.embed = torch.zeros(V, V, dtype=torch.bfloat16)
        eng.lm_head = torch.eye(V, dtype=torch.bfloat16)
        eng.norm_weight = None
        eng.hc_head_fn = None
        eng._get_layer_weights = lambda i: {}
        ids = [5, 9, 13]
        lg = torch.zeros(3, V)
        lg[0, 9 if n_want >= 1 else 10] = 1.0    # predicts combined[1] = 9 or not
        lg[1, 13 if n_want >= 2 else 14] = 1.0
        lg[2, 20] = 1.0

        def fwd(h, lw, i, ids_, lg=lg):
            ls, comp = eng.layer_states[i], eng._compressors[i]
            st = {"kv": ls.kv_latent_cache, "cdata": ls.compressed_kv_data, "cidx": ls.compressed_kv_idx,
                  "comp": (comp.accumulated, comp.kv_state, comp.score_state)}
            VS.forward_mutation(st, [int(x) for x in ids_.reshape(-1)], i)
            ls.kv_latent_cache, ls.compressed_kv_data, ls.compressed_kv_idx = st["kv"], st["cdata"], st["cidx"]
            comp.accumulated, comp.kv_state, comp.score_state = st["comp"]
            return lg.view(1, 3, 1, V).to(torch.bfloat16), set()
        eng._forward_layer = fwd
        n, _ = eng._mtp_verify_batched(torch.tensor([ids[1:]]), 0.0, main_pred_id=torch.tensor([[ids[0]]]))
        assert n == n_want
        out[f"vs{case}_n"] = np.array([n, eng._global_pos], dtype=np.int64)
        for l, ls in eng.layer_states.items():
            comp = eng._compressors[l]
            out[f"vs{case}_kv{l}"] = _bf16_np(ls.kv_latent_cache)
            out[f"vs{case}_cdata{l}"] = _bf16_np(ls.compressed_kv_data)
            out[f"vs{case}_cidx{l}"] = ls.compressed_kv_idx.numpy()
            out[f"vs{case}_acc{l}"] = np.array([comp.accumulated], dtype=np.int64)
            out[f"vs{case}_kvs{l}"] = comp.kv_state.numpy()
            out[f"vs{case}_scs{l}"] = comp.score_state.numpy()


def main():
    sys.path.insert(0, str(_ref_path()))
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    out = {}
    gen_router(out)
    gen_hash(out)
    gen_accept(out)
    gen_permute(out)
    gen_moe(out)
    gen_mtp(out)
    gen_verify_state(out)
    np.savez_compressed(HERE / "golden.npz", **out)
    print("wrote", HERE / "golden.npz", len(out), "arrays")


if __name__ == "__main__":
    main()
