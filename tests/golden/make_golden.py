"""Write the golden fixtures of this directory by running the REFERENCE code on seeded inputs.

Usage (only where the reference checkout exists; the GPU box does not have it):
    DIMMERKV_REFERENCE=/path/to/Dimmer-KV python tests/golden/make_golden.py [fixture ...]
(no names: every fixture; names such as ``encode``, ``codes``, ``storage``, ``logits``, ``f16`` or ``tiny``:
only those).

Every array saved here is produced by the reference's own functions (scripts/progressive.py,
scripts/kvtc.py, scripts/compressed_attention.py, scripts/dimmer.py, scripts/methods.py,
scripts/fit_kvtc.py) on the seeded tiny model of ``tinymodel.py``. Tests compare the numpy
oracle and the CUDA path against these arrays; nothing at test time imports the reference.
"""

from __future__ import annotations

import os
import sys
import tempfile
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
if "DIMMERKV_REFERENCE" not in os.environ:
    raise SystemExit("set DIMMERKV_REFERENCE to the reference checkout (the directory holding scripts/)")
REF = Path(os.environ["DIMMERKV_REFERENCE"]) / "scripts"
sys.path.insert(0, str(REF))

import compressed_attention  # noqa: E402  (reference)
import dimmer  # noqa: E402
import kvtc  # noqa: E402
import progressive  # noqa: E402
from common import build_cache  # noqa: E402
from fit_kvtc import TARGETS, build_ladder  # noqa: E402
from methods import Methods  # noqa: E402

import tinymodel as tm  # noqa: E402


def bits16(t: torch.Tensor) -> np.ndarray:
    """bf16 / f16 tensor -> uint16 bit patterns."""
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def codes_fixture(out: Path) -> None:
    g = torch.Generator().manual_seed(5)
    coeff = torch.randn(96, 512, generator=g) * torch.logspace(1, -3, 512)[None]
    coeff[3, :64] = 0.0           # constant group (span rounds to 0)
    coeff[4, 64:128] = 0.25       # constant non-zero group
    coeff[5, 128:192] *= 1e-7     # tiny span
    codes, low, span = progressive.quantize8(coeff, 64)
    planes = torch.randint(0, 9, (96, 8), generator=g)
    deq = progressive.dequantize(codes, low, span, planes)
    bits = torch.tensor([8, 4, 4, 2, 2, 2, 0, 0])
    ladder = kvtc.quantize_groups(coeff, bits, 64)
    np.savez_compressed(
        out / "codes.npz", coeff=coeff.numpy(), codes=codes.numpy(), low=bits16(low), span=bits16(span),
        planes=planes.numpy(), deq=deq.numpy(),
        ladder_bits=bits.numpy(), ladder=ladder.numpy(),
    )


def allocator_fixture(out: Path) -> None:
    g = torch.Generator().manual_seed(8)
    middle, levels = 50, 6
    errors = torch.rand(2 * middle, levels, generator=g).sort(dim=1, descending=True).values
    level_bytes = torch.tensor([10, 20, 40, 80, 160, 320, 12, 24, 48, 96, 192, 384])
    chosen = kvtc.allocate_rungs(errors, level_bytes, middle, 8000)
    np.savez_compressed(out / "allocator.npz", errors=errors.numpy(), level_bytes=level_bytes.numpy(),
                        middle=middle, budget=8000, chosen=chosen.numpy())


def encode_fixture(out: Path) -> None:
    """The error side of ProgressiveCodec.encode (progressive.py:150-163) on seeded coefficients: the
    reference's quantize8 / dequantize / build_order, and encode's table, gather and sums written out
    line by line (they are inline in encode, not a function of their own)."""
    g = torch.Generator().manual_seed(21)
    scales = torch.logspace(1.5, -3, 1024)[None]
    calib = torch.randn(200, 1024, generator=g) * scales
    coeff = torch.randn(300, 1024, generator=g) * scales
    coeff[7, :64] = 0.0             # constant group: span rounds to 0
    coeff[8, 64:128] = -1.5         # constant non-zero group
    coeff[9, 128:192] *= 1e-6       # tiny span
    coeff[10, 192:256] *= 1e3       # wide span (still inside the f16 range)
    order = progressive.build_order(calib, 64, TARGETS, 2 * 1024)
    codes, low, span = progressive.quantize8(coeff, 64)
    middle, groups = coeff.shape[0], 16
    grouped = coeff.view(middle, -1, 64)
    table = torch.stack([
        (grouped - progressive.dequantize(codes, low, span, torch.full((1, groups), m)).view_as(grouped))
        .square().sum(dim=-1)
        for m in range(progressive.PLANES + 1)
    ], dim=-1)
    rung_planes = order.planes[order.rungs].long().T
    rung_sum = table.gather(2, rung_planes[None].expand(middle, -1, -1)).sum(dim=1)
    token_energy = coeff.square().sum(dim=1)
    energy = token_energy.mean().clamp_min(1e-12)
    np.savez_compressed(
        out / "encode.npz", coeff=coeff.numpy(), rung_planes=order.planes[order.rungs].numpy(),
        rungs=np.array(order.rungs), codes=codes.numpy(), low=bits16(low), span=bits16(span),
        table=table.numpy(), rung_sum=rung_sum.numpy(), token_energy=token_energy.numpy(),
        rung_error=(rung_sum / energy).numpy(),
    )


def storage_fixture(out: Path, methods, keys, values, scores) -> None:
    """kvtc_storage.encode_bytes / decode_bytes of the tiny model's dkvtc caches at two budgets, the
    second one high enough that some tokens take the ladder's exact rung (the reference's byte format,
    kvtc_storage.py:42-135)."""
    import kvtc_storage  # reference

    fixture = {}
    for tag, name in (("lo", "dkvtc@0.1:snap:floor1"), ("hi", "dkvtc@0.6:snap:floor1")):
        with torch.inference_mode():
            methods.apply(name, keys, values, scores)
            codec = methods.codec("kvtc")
            data = kvtc_storage.encode_bytes(codec, keys, values, codec.last_choice, tm.RECENT)
            dec_keys, dec_values = kvtc_storage.decode_bytes(codec, data, dtype=torch.float32)
        fixture.update({
            f"{tag}_name": name, f"{tag}_data": np.frombuffer(data, dtype=np.uint8),
            f"{tag}_choice_key": codec.last_choice["key"].numpy(), f"{tag}_choice_value": codec.last_choice["value"].numpy(),
            # Layer 0, KV heads 0-1 of the restored caches (float32), to keep the file small.
            f"{tag}_keys": dec_keys[0][0, :2].numpy(), f"{tag}_values": dec_values[0][0, :2].numpy(),
        })
    fixture["exact_rung"] = len(methods.codec("kvtc").streams["key"].rung_bytes)
    np.savez_compressed(out / "storage.npz", **fixture)


GEOMETRY_3B = dict(tm.TINY, hidden_size=768, num_attention_heads=24, head_dim=128)  # Llama-3.2-3B heads, tiny model
GEOMETRY_3B_TOKENS, GEOMETRY_3B_GROUPS, GEOMETRY_3B_BASIS_SEED = 230, 6, 500


def geometry3b_fixture(out: Path) -> None:
    """The reference's CompressedContext (_keys, attend) at the Llama-3.2-3B head geometry (8 KV heads of
    128, 24 query heads, GQA 3) on a 2-layer random-init model, over synthetic progressive codes
    (quantize8 of seeded coefficients, per-token plane counts {0,1,2,4,6,8} on the first groups) fed
    through a codec shim; fp32 and bf16 runs at q = 1 and 4. The bases are rebuilt from their seed by
    the tests (tinymodel.seeded_basis)."""
    from transformers import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(4321)
    model = LlamaForCausalLM(LlamaConfig(**GEOMETRY_3B)).float().eval()
    layers, heads, dim = GEOMETRY_3B["num_hidden_layers"], GEOMETRY_3B["num_key_value_heads"], GEOMETRY_3B["head_dim"]
    q_heads = GEOMETRY_3B["num_attention_heads"]
    features, tokens, used = layers * heads * dim, GEOMETRY_3B_TOKENS, GEOMETRY_3B_GROUPS
    start, end = tm.SINKS, tokens - tm.RECENT
    middle = end - start
    g = torch.Generator().manual_seed(77)
    fixture = {"span": np.array([start, end]), "tokens": tokens, "groups_used": used}
    shim = types.SimpleNamespace(layers=layers, heads=heads, head_dim=dim, device=torch.device("cpu"),
                                 last_span=(start, end), streams={}, last_choice={}, last_coefficients={})
    for index, kind in enumerate(("key", "value")):
        coeff = torch.randn(middle, features, generator=g) * torch.logspace(0, -2, features)[None]
        codes, low, span = progressive.quantize8(coeff, tm.GROUP)
        pick = torch.multinomial(torch.tensor([.05, .35, .25, .2, .1, .05]), middle, replacement=True, generator=g)
        m = torch.tensor([0, 1, 2, 4, 6, 8])[pick]
        planes = torch.zeros(middle, features // tm.GROUP, dtype=torch.long)
        planes[:, :used] = m[:, None]
        basis = tm.seeded_basis(features, features, GEOMETRY_3B_BASIS_SEED + index)
        mean = torch.randn(features, generator=g) * 0.1
        shim.streams[kind] = types.SimpleNamespace(mean=mean, basis=basis)
        shim.last_choice[kind] = m
        shim.last_coefficients[kind] = progressive.dequantize(codes, low, span, planes)
        fixture[f"codes_{kind}"] = codes[:, :used].numpy()
        fixture[f"low_{kind}"] = bits16(low[:, :used])
        fixture[f"span_{kind}"] = bits16(span[:, :used])
        fixture[f"planes_{kind}"] = m.numpy()
        fixture[f"mean_{kind}"] = mean.numpy()
    keys = [torch.randn(1, heads, tokens, dim, generator=g).to(torch.bfloat16) for _ in range(layers)]
    values = [torch.randn(1, heads, tokens, dim, generator=g).to(torch.bfloat16) for _ in range(layers)]
    fixture["exact_keys"] = np.stack([bits16(torch.cat([k[..., :start, :], k[..., end:, :]], dim=2)[0]) for k in keys])
    fixture["exact_values"] = np.stack([bits16(torch.cat([v[..., :start, :], v[..., end:, :]], dim=2)[0]) for v in values])
    cos, sin = kvtc.rope_tables(model, tokens, "cpu")
    fixture["cos"], fixture["sin"] = cos.float().numpy(), sin.float().numpy()
    queries = {q: torch.randn(1, q_heads, q, dim, generator=g).to(torch.bfloat16) for q in (1, 4)}
    news = {q: (torch.randn(1, heads, q, dim, generator=g).to(torch.bfloat16),
                torch.randn(1, heads, q, dim, generator=g).to(torch.bfloat16)) for q in (1, 4)}
    for q in (1, 4):
        fixture[f"query_q{q}"] = queries[q].float().numpy()
        fixture[f"newk_q{q}"] = news[q][0].float().numpy()
        fixture[f"newv_q{q}"] = news[q][1].float().numpy()
    module = types.SimpleNamespace(layer_idx=0, num_key_value_groups=q_heads // heads)
    with torch.inference_mode():
        for dtype, tag in ((torch.bfloat16, "bf16"), (torch.float32, "f32")):
            ctx = compressed_attention.CompressedContext(shim, [k.to(dtype) for k in keys], [v.to(dtype) for v in values],
                                                         model, dtype=dtype)
            for layer in range(layers):
                module.layer_idx = layer
                ex = ctx.exact_cache.layers[layer]
                for q in (1, 4):
                    k = torch.cat([ex.keys, news[q][0].to(dtype)], dim=2)
                    v = torch.cat([ex.values, news[q][1].to(dtype)], dim=2)
                    mask = None
                    if q > 1:
                        e = k.shape[2]
                        mask = torch.zeros(1, 1, q, e, dtype=dtype)
                        causal = torch.triu(torch.ones(q, q, dtype=torch.bool), 1)
                        mask[0, 0, :, e - q:][causal] = torch.finfo(dtype).min
                    out_, _ = ctx.attend(module, queries[q].to(dtype), k, v, mask, dim ** -0.5)
                    fixture[f"{tag}_attend_l{layer}_q{q}"] = out_.float().numpy()
            if dtype == torch.float32:
                fixture["f32_keys_l0"] = ctx._keys(0).numpy()
    np.savez_compressed(out / "geometry3b.npz", **fixture)


def logits_fixture(out: Path, methods, model, keys, values, scores, tokens: int) -> None:
    """First-step logits and greedy replies of the reference's greedy_answer (compressed_attention.py:140-169)
    over dkvtc@0.1:snap:floor1 codes, once in bf16 (model, cache and context, as tiny_dkvtc's greedy_direct)
    and once in float32: the float32 run bounds the reference's own bf16 rounding for the logit tests."""
    rng_state = torch.random.get_rng_state()  # building a model reseeds torch; later fixtures keep their draws
    try:
        name = "dkvtc@0.1:snap:floor1"
        tok = types.SimpleNamespace(eos_token_id=-1, all_special_ids=[],
                                    decode=lambda ids, skip_special_tokens=True: " ".join(map(str, ids)))
        tail = tm.question_ids()
        result = {"name": name, "tail": tail.numpy()}
        with torch.inference_mode():
            methods.apply(name, keys, values, scores)
            codec = methods.codec("kvtc")
            model32 = tm.build_model(torch.float32)
            dimmer.install(model32)
            for tag, dtype, m in (("bf16", torch.bfloat16, model), ("f32", torch.float32, model32)):
                ctx = compressed_attention.CompressedContext(codec, [k.to(dtype) for k in keys],
                                                             [v.to(dtype) for v in values], m, dtype=dtype)
                exact = build_cache([l.keys.clone() for l in ctx.exact_cache.layers],
                                    [l.values.clone() for l in ctx.exact_cache.layers], m)
                text, logits = compressed_attention.greedy_answer(m, tok, ctx, exact, tail[None], tokens, 4,
                                                                  stop_at_eos=False)
                result[f"logits_{tag}"] = logits.float().numpy()
                result[f"greedy_{tag}"] = np.array([int(x) for x in text.split()])
        np.savez_compressed(out / "tiny_logits.npz", **result)
    finally:
        torch.random.set_rng_state(rng_state)


def f16_fixture(out: Path, methods, model, keys, values, scores, tokens: int) -> None:
    """The reference's CompressedContext in float16 (its default dtype, compressed_attention.py:34-35) on the
    two entry points' codes: attention outputs of both layers at q = 1 and 4 (the same queries, new tokens and
    masks as tiny_dkvtc / tiny_prog), and greedy_answer's first-step logits and reply with the model in
    float16 over the dkvtc codes."""
    rng_state = torch.random.get_rng_state()
    try:
        cfg = model.config
        layers, heads, dim = cfg.num_hidden_layers, cfg.num_key_value_heads, cfg.head_dim
        g = torch.Generator().manual_seed(21)  # the draws of main(): same queries and new tokens
        module = types.SimpleNamespace(num_key_value_groups=cfg.num_attention_heads // heads)
        queries = {q: torch.randn(1, cfg.num_attention_heads, q, dim, generator=g) for q in (1, 4)}
        news = {q: (torch.randn(1, heads, q, dim, generator=g), torch.randn(1, heads, q, dim, generator=g))
                for q in (1, 4)}
        dtype = torch.float16
        result = {}

        def attend_all(ctx, tag):
            for layer in range(layers):
                module.layer_idx = layer
                ex = ctx.exact_cache.layers[layer]
                for q in (1, 4):
                    k = torch.cat([ex.keys, news[q][0].to(dtype)], dim=2)
                    v = torch.cat([ex.values, news[q][1].to(dtype)], dim=2)
                    mask = None
                    if q > 1:
                        e = k.shape[2]
                        mask = torch.zeros(1, 1, q, e, dtype=dtype)
                        causal = torch.triu(torch.ones(q, q, dtype=torch.bool), 1)
                        mask[0, 0, :, e - q:][causal] = torch.finfo(dtype).min
                    out_, _ = ctx.attend(module, queries[q].to(dtype), k, v, mask, dim ** -0.5)
                    result[f"{tag}_f16_attend_l{layer}_q{q}"] = out_.float().numpy()

        with torch.inference_mode():
            methods.apply("dkvtc@0.1:snap:floor1", keys, values, scores)
            codec = methods.codec("kvtc")
            ctx = compressed_attention.CompressedContext(codec, [k.to(dtype) for k in keys],
                                                         [v.to(dtype) for v in values], model)
            assert ctx.dtype == dtype  # the reference's default
            attend_all(ctx, "dkvtc")
            pcodec = methods.codec("prog")
            stored = pcodec.encode(keys, values, 0.1, tm.RECENT, None)
            shim = types.SimpleNamespace(layers=layers, heads=heads, head_dim=dim, device=torch.device("cpu"),
                                         last_span=(stored.start, stored.end), streams={}, last_choice={},
                                         last_coefficients={})
            for kind in ("key", "value"):
                s = stored.stores[kind]
                planes = pcodec.orders[kind].planes[s.hot_pieces]
                shim.streams[kind] = pcodec.base.streams[kind]
                shim.last_choice[kind] = s.hot_pieces
                shim.last_coefficients[kind] = progressive.dequantize(s.codes, s.low, s.span, planes)
            ctx = compressed_attention.CompressedContext(shim, [k.to(dtype) for k in keys],
                                                         [v.to(dtype) for v in values], model)
            attend_all(ctx, "prog")
            # greedy_answer with the model in float16 over the dkvtc codes
            methods.apply("dkvtc@0.1:snap:floor1", keys, values, scores)
            model16 = tm.build_model(dtype)
            dimmer.install(model16)
            ctx = compressed_attention.CompressedContext(codec, [k.to(dtype) for k in keys],
                                                         [v.to(dtype) for v in values], model16)
            exact = build_cache([l.keys.clone() for l in ctx.exact_cache.layers],
                                [l.values.clone() for l in ctx.exact_cache.layers], model16)
            tok = types.SimpleNamespace(eos_token_id=-1, all_special_ids=[],
                                        decode=lambda ids, skip_special_tokens=True: " ".join(map(str, ids)))
            tail = tm.question_ids()
            text, logits = compressed_attention.greedy_answer(model16, tok, ctx, exact, tail[None], tokens, 4,
                                                              stop_at_eos=False)
            result.update(tail=tail.numpy(), logits_f16=logits.float().numpy(),
                          greedy_f16=np.array([int(x) for x in text.split()]))
        np.savez_compressed(out / "tiny_f16.npz", **result)
    finally:
        torch.random.set_rng_state(rng_state)


def main() -> None:
    out = HERE
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    only = sys.argv[1:]
    standalone = {"codes", "allocator", "encode", "geometry3b"}  # fixtures that need no prefilled context
    for name in only:
        if name in standalone:  # e.g. `make_golden.py encode`: write just the named fixtures
            globals()[f"{name}_fixture"](out)
    if only and not (set(only) - standalone):
        return
    if not only:
        codes_fixture(out)
        allocator_fixture(out)
        encode_fixture(out)
        geometry3b_fixture(out)

    model = tm.build_model(torch.bfloat16)
    dimmer.install(model)
    cfg = model.config
    layers, heads, dim = cfg.num_hidden_layers, cfg.num_key_value_heads, cfg.head_dim
    features = layers * heads * dim
    ids = tm.context_ids()
    with torch.inference_mode():
        cache, scores = dimmer.prefill_with_scores(model, ids)
    keys = [l.keys.clone() for l in cache.layers]
    values = [l.values.clone() for l in cache.layers]
    tokens = keys[0].shape[2]
    cos, sin = kvtc.rope_tables(model, tokens, "cpu")
    start, end = tm.SINKS, tokens - tm.RECENT

    # Synthetic calibration files (full-rank seeded bases; mean over this context's middle tokens).
    saved = {"model": "tiny", "layers": layers, "heads": heads, "head_dim": dim, "group": tm.GROUP, "sinks": tm.SINKS}
    orders = {"model": "tiny", "kvtc": "kvtc.pt"}
    bases = {}
    for index, (kind, tensors) in enumerate((("key", keys), ("value", values))):
        basis = tm.seeded_basis(features, features, tm.SEED_BASIS + index)
        bases[kind] = basis
        matrix = kvtc.token_matrix([kvtc.derotate(t, cos, sin) for t in tensors] if kind == "key" else tensors)
        mean = matrix[start:end].mean(0)
        coefficients = (matrix[start:end] - mean) @ basis
        rungs, sizes = build_ladder(coefficients, tm.GROUP, features * 2)
        saved[kind] = {"mean": mean, "basis": basis, "rungs": rungs, "rung_bytes": sizes}
        order = progressive.build_order(coefficients, tm.GROUP, TARGETS, features * 2)
        orders[kind] = {"planes": order.planes, "prefix_bytes": order.prefix_bytes, "rungs": order.rungs}
    tmp = Path(tempfile.mkdtemp())
    torch.save(saved, tmp / "kvtc.pt")
    torch.save(orders, tmp / "progressive.pt")
    methods = Methods("tiny", tmp / "none", tmp / "none", torch.device("cpu"), tm.RECENT, model=model,
                      kvtc=tmp / "kvtc.pt", progressive=tmp / "progressive.pt")
    if not only or "storage" in only:
        storage_fixture(out, methods, keys, values, scores)
    if not only or "logits" in only:
        logits_fixture(out, methods, model, keys, values, scores, tokens)
    if not only or "f16" in only:
        f16_fixture(out, methods, model, keys, values, scores, tokens)
    if only and "tiny" not in only:
        return

    inputs = dict(ids=ids.numpy(), keys=np.stack([bits16(k[0]) for k in keys]),
                  values=np.stack([bits16(v[0]) for v in values]),
                  snap=torch.stack(scores["snap"]).float().numpy(),
                  checksum=tm.model_checksum(model),
                  basis_checksum=np.array([float(bases[k].double().sum()) for k in ("key", "value")]),
                  mean_key=saved["key"]["mean"].numpy(), mean_value=saved["value"]["mean"].numpy(),
                  cos=cos.numpy(), sin=sin.numpy())
    for kind in ("key", "value"):
        inputs[f"rungs_{kind}"] = saved[kind]["rungs"].numpy()
        inputs[f"rung_bytes_{kind}"] = np.array(saved[kind]["rung_bytes"])
        inputs[f"order_planes_{kind}"] = orders[kind]["planes"].numpy()
        inputs[f"order_prefix_{kind}"] = orders[kind]["prefix_bytes"].numpy()
        inputs[f"order_rungs_{kind}"] = np.array(orders[kind]["rungs"])
    np.savez_compressed(out / "tiny_inputs.npz", **inputs)

    g = torch.Generator().manual_seed(21)
    module = types.SimpleNamespace(num_key_value_groups=cfg.num_attention_heads // heads)
    queries = {q: torch.randn(1, cfg.num_attention_heads, q, dim, generator=g) for q in (1, 4)}
    news = {q: (torch.randn(1, heads, q, dim, generator=g), torch.randn(1, heads, q, dim, generator=g)) for q in (1, 4)}

    def attend_all(ctx, dtype):
        result = {}
        for layer in range(layers):
            module.layer_idx = layer
            ex = ctx.exact_cache.layers[layer]
            for q in (1, 4):
                k = torch.cat([ex.keys, news[q][0].to(dtype)], dim=2)
                v = torch.cat([ex.values, news[q][1].to(dtype)], dim=2)
                mask = None
                if q > 1:
                    e = k.shape[2]
                    mask = torch.zeros(1, 1, q, e, dtype=dtype)
                    causal = torch.triu(torch.ones(q, q, dtype=torch.bool), 1)
                    mask[0, 0, :, e - q:][causal] = torch.finfo(dtype).min
                out_, _ = ctx.attend(module, queries[q].to(dtype), k, v, mask, dim ** -0.5)
                result[f"attend_l{layer}_q{q}"] = out_.float().numpy()
            if dtype == torch.bfloat16 or layer == 0:
                rebuilt = ctx._keys(layer)
                result[f"keys_l{layer}"] = bits16(rebuilt) if dtype == torch.bfloat16 else rebuilt.numpy()
        return result

    shared_attend_inputs = {f"query_q{q}": queries[q].numpy() for q in (1, 4)}
    for q in (1, 4):
        shared_attend_inputs[f"newk_q{q}"] = news[q][0].numpy()
        shared_attend_inputs[f"newv_q{q}"] = news[q][1].numpy()

    # ---- dkvtc@b:snap:floor1 (the kvtc ladder entry point)
    name = "dkvtc@0.1:snap:floor1"
    with torch.inference_mode():
        compressed = methods.apply(name, keys, values, scores)
        codec = methods.codec("kvtc")
        fixture = {"name": name, "used_bytes": compressed.used_bytes,
                   "span": np.array(codec.last_span)}
        for kind in ("key", "value"):
            fixture[f"choice_{kind}"] = codec.last_choice[kind].numpy()
            fixture[f"coeff_{kind}"] = codec.last_coefficients[kind].numpy()
        for dtype, tag in ((torch.bfloat16, "bf16"), (torch.float32, "f32")):
            ctx = compressed_attention.CompressedContext(codec, [k.to(dtype) for k in keys],
                                                         [v.to(dtype) for v in values], model, dtype=dtype)
            for key, val in attend_all(ctx, dtype).items():
                fixture[f"{tag}_{key}"] = val
            fixture[f"{tag}_code_bytes"] = ctx.code_bytes()
        # Direct greedy answer over codes vs the rebuilt cache (test_compressed_attention.py:89-98).
        tail = tm.question_ids()
        ctx = compressed_attention.CompressedContext(codec, keys, values, model, dtype=torch.bfloat16)
        exact = build_cache([l.keys.clone() for l in ctx.exact_cache.layers],
                            [l.values.clone() for l in ctx.exact_cache.layers], model)
        tok = types.SimpleNamespace(eos_token_id=-1, all_special_ids=[], decode=lambda ids, skip_special_tokens=True: " ".join(map(str, ids)))
        text_d, logits_d = compressed_attention.greedy_answer(model, tok, ctx, exact, tail[None], tokens, 4,
                                                              stop_at_eos=False)
        full = build_cache([k.clone() for k in compressed.keys], [v.clone() for v in compressed.values], model)
        text_r, logits_r = compressed_attention.greedy_answer(model, tok, None, full, tail[None], tokens, 4,
                                                              stop_at_eos=False)
        fixture.update(tail=tail.numpy(), greedy_direct=np.array([int(x) for x in text_d.split()]),
                       greedy_rebuilt=np.array([int(x) for x in text_r.split()]),
                       logits_direct=logits_d.numpy(), logits_rebuilt=logits_r.numpy())
    fixture.update(shared_attend_inputs)
    np.savez_compressed(out / "tiny_dkvtc.npz", **fixture)

    # ---- prog@b:r<frac> (progressive codec, hot tier, question-time refine)
    name, budget, fraction = "prog@0.1:r0.05", 0.1, 0.05
    with torch.inference_mode():
        pcodec = methods.codec("prog")
        stored = pcodec.encode(keys, values, budget, tm.RECENT, None)
        fixture = {"name": name, "hot_bytes": stored.hot_bytes, "cold_bytes": stored.cold_bytes,
                   "budget_bytes": stored.budget_bytes, "span": np.array([stored.start, stored.end])}
        for kind in ("key", "value"):
            s = stored.stores[kind]
            fixture[f"codes_{kind}"] = s.codes.numpy()
            fixture[f"low_{kind}"] = bits16(s.low)
            fixture[f"lowspan_{kind}"] = bits16(s.span)
            fixture[f"hot_pieces_{kind}"] = s.hot_pieces.numpy()
        hot_keys, hot_values = stored.hot()
        importance = progressive.question_importance(model, hot_keys, hot_values, tm.question_ids(), tokens)
        middle = stored.end - stored.start
        count = max(1, int(round(fraction * middle)))
        top = importance[stored.start:stored.end].topk(count).indices + stored.start
        ref_keys, ref_values, fetched = stored.refine(hot_keys, hot_values, top)
        fixture.update(importance=importance.float().numpy(), top=top.numpy(), fetched=fetched, count=count)
        rows = top.sort().values
        fixture["refined_keys"] = np.stack([bits16(k[0][:, rows]) for k in ref_keys])
        fixture["refined_values"] = np.stack([bits16(v[0][:, rows]) for v in ref_values])
        fixture["hot_keys_rows"] = np.stack([bits16(k[0][:, rows]) for k in hot_keys])
        # Direct attention over the hot progressive codes: a codec shim exposing the fields that
        # CompressedContext reads (compressed_attention.py:36-54).
        shim = types.SimpleNamespace(layers=layers, heads=heads, head_dim=dim, device=torch.device("cpu"),
                                     last_span=(stored.start, stored.end), streams={}, last_choice={},
                                     last_coefficients={})
        for kind in ("key", "value"):
            s = stored.stores[kind]
            planes = pcodec.orders[kind].planes[s.hot_pieces]
            shim.streams[kind] = pcodec.base.streams[kind]
            shim.last_choice[kind] = s.hot_pieces
            shim.last_coefficients[kind] = progressive.dequantize(s.codes, s.low, s.span, planes)
        for dtype, tag in ((torch.bfloat16, "bf16"), (torch.float32, "f32")):
            ctx = compressed_attention.CompressedContext(shim, [k.to(dtype) for k in keys],
                                                         [v.to(dtype) for v in values], model, dtype=dtype)
            for key, val in attend_all(ctx, dtype).items():
                fixture[f"{tag}_{key}"] = val
    fixture.update(shared_attend_inputs)
    np.savez_compressed(out / "tiny_prog.npz", **fixture)
    for f in sorted(out.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
