"""Generate the golden fixtures in this directory by running the reference.

Run from the repository root in a checkout that has the reference sources:

    python tests/golden/make_golden.py /path/to/reference/src

It imports the reference package (``anchorkv``) from that path, runs its codec
(``backend.quantize_tensor``, ``packed_decode.pack_page``), its block stores
(``DeclarativeKVCache``, ``PagedLayer``), its dense decode path
(``dense_attention`` / ``materialize_visible`` + SDPA) and its ``requantize-demo``
report on seeded inputs, and writes:

* ``codec.npz`` + ``codec.json`` -- quantizer inputs, payloads, scales, dequantised values;
* ``attention.npz`` + ``attention.json`` -- decode outputs and sha256 digests of
  the dense K/V the reference attended over;
* ``demo.json`` -- the ``requantize-demo`` storage report (INT4 and INT8);
* ``declarative.npz`` + ``declarative.json`` -- the block store on page-format
  scenarios: visibility, positions, storage reports, digests of the dense K/V
  and per-layer decode outputs.

Nothing at test time reads the reference; the tests read these files.
"""

from __future__ import annotations

import json
import math
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import workloads as W  # noqa: E402


def _np(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy()  # stored as raw bits
    return t.numpy()


def _store_input(arrays, x: torch.Tensor) -> str:
    """Store each distinct input once, keyed by its digest."""
    key = "in_" + W.sha256(x)[:16]
    arrays.setdefault(key, _np(x))
    return key


def codec_cases():
    cases = []
    torch.manual_seed(7)
    unit = torch.randn(1, 2, 10, 8, dtype=torch.float32)
    for bits in (8, 4):
        cases.append((f"unit_f32_b{bits}_g16", unit, bits, 16))
    pad = torch.randn(2, 3, 5, 7, generator=W.generator(21))
    for bits in (8, 4):
        for group in (16, 10, 64):
            cases.append((f"pad_f32_b{bits}_g{group}", pad, bits, group))
    slab = W.outlier_kv(31, (1, 8, 16, 128), signed=True)
    for bits in (8, 4):
        for group in (2048, 64):
            cases.append((f"slab_f16_b{bits}_g{group}", slab, bits, group))
    bf = torch.randn(1, 4, 16, 64, generator=W.generator(41)).to(torch.bfloat16)
    for bits in (8, 4):
        cases.append((f"bf16_b{bits}_g64", bf, bits, 64))
    zeros = torch.zeros(1, 1, 4, 8)
    for bits in (8, 4):
        cases.append((f"zeros_b{bits}_g16", zeros, bits, 16))
    tiny32 = torch.full((1, 2, 16, 8), 1e-7)
    tiny16 = tiny32.half()
    for bits in (8, 4):
        cases.append((f"tiny_f32_b{bits}_g16", tiny32, bits, 16))
        cases.append((f"tiny_f16_b{bits}_g16", tiny16, bits, 16))
    sub = (torch.randn(1, 2, 16, 64, generator=W.generator(51)) * 1e-5).half()
    for bits in (8, 4):
        cases.append((f"subnormal_b{bits}_g64", sub, bits, 64))
    ties4 = torch.tensor([7, 0.5, 1.5, 2.5, 3.5, -0.5, -1.5, -2.5, -3.5,
                          4.5, 5.5, 6.5, -4.5, -5.5, -6.5, 0.0]).reshape(1, 1, 2, 8)
    cases.append(("ties_b4_g16", ties4, 4, 16))
    ties8 = torch.cat([torch.tensor([127.0]), torch.arange(-62, 63, dtype=torch.float32) + 0.5,
                       torch.tensor([-127.0, 0.0])]).reshape(1, 1, 8, 16)
    cases.append(("ties_b8_g128", ties8, 8, 128))
    large = (torch.randn(1, 2, 16, 32, generator=W.generator(61)) * 20000).clamp(-60000, 60000).half()
    for bits in (8, 4):
        cases.append((f"large_b{bits}_g64", large, bits, 64))
    partial = W.outlier_kv(71, (1, 8, 6, 128))
    for bits in (8, 4):
        cases.append((f"partial_block_b{bits}_g2048", partial, bits, 2048))
    odd = torch.randn(1, 1, 3, 5, generator=W.generator(81))
    for bits in (8, 4):
        cases.append((f"odd_b{bits}_g4", odd, bits, 4))
    return cases


def page_cases():
    cases = []
    torch.manual_seed(11)
    source = torch.randn(2, 16, 128).half()
    for bits in (4, 8, 16):
        cases.append((f"unit_b{bits}_g64", source, bits, 64))
    tiny = torch.full_like(source, 1e-7)
    for bits in (4, 8):
        cases.append((f"tiny_b{bits}_g64", tiny, bits, 64))
    out = W.outlier_kv(91, (8, 16, 128), signed=True)
    for bits in (4, 8):
        for group in (32, 64, 128):
            cases.append((f"outlier_b{bits}_g{group}", out, bits, group))
    d64 = torch.randn(2, 16, 64, generator=W.generator(101)).half()
    for bits in (4, 8):
        cases.append((f"d64_b{bits}_g64", d64, bits, 64))
    cases.append(("zeros_b4_g64", torch.zeros(2, 16, 128).half(), 4, 64))
    f32 = torch.randn(2, 16, 128, generator=W.generator(111)) * 3
    cases.append(("f32_b4_g64", f32, 4, 64))
    return cases


def build_codec(anchorkv):
    from anchorkv.backend import quantize_tensor
    from anchorkv.packed_decode import pack_page
    from anchorkv.policy import CacheMode

    mode_of = {8: CacheMode.INT8, 4: CacheMode.INT4}
    arrays, meta = {}, {"tensor": [], "page": []}
    for name, x, bits, group in codec_cases():
        packed = quantize_tensor(x, mode_of[bits], group_size=group)
        restored = packed.dequantize()
        key = f"t_{name}"
        source = _store_input(arrays, x)
        arrays[key + "_payload"] = _np(packed.payload)
        arrays[key + "_scales"] = _np(packed.scales)
        arrays[key + "_deq"] = _np(restored)
        meta["tensor"].append({"name": name, "bits": bits, "group": group, "input": source,
                               "dtype": str(x.dtype).replace("torch.", ""),
                               "shape": list(x.shape), "stored_bytes": packed.stored_bytes})
    for name, x, bits, group in page_cases():
        page = pack_page(x, bits, group)
        key = f"p_{name}"
        source = _store_input(arrays, x)
        arrays[key + "_payload"] = _np(page.data)
        if page.scales is not None:
            arrays[key + "_scales"] = _np(page.scales)
        arrays[key + "_dense"] = _np(page.dense())
        meta["page"].append({"name": name, "bits": bits, "group": group, "input": source,
                             "dtype": str(x.dtype).replace("torch.", ""),
                             "shape": list(x.shape), "nbytes": page.nbytes})
    np.savez_compressed(HERE / "codec.npz", **arrays)
    (HERE / "codec.json").write_text(json.dumps(meta, indent=1))


def build_attention(anchorkv):
    from anchorkv.backend import DeclarativeKVCache, SegmentRole
    from anchorkv.packed_decode import PagedLayer, dense_attention
    from anchorkv.policy import CacheMode

    arrays, meta = {}, {"gate": [], "parity": []}
    for dim in W.GATE_DIMS:
        for length in W.GATE_LENGTHS:
            for bits in W.GATE_BITS:
                seed = W.gate_seed(dim, length, bits)
                q, k, v = W.gate_workload(dim, length, seed)
                layer = PagedLayer(2, dim, 128, archive_bits=bits, protected=(0,),
                                   recent_pages=1, device="cpu")
                for begin in range(0, length, 7):
                    layer.append(k[:, :, begin:begin + 7], v[:, :, begin:begin + 7])
                out = dense_attention(q, layer, dim ** -0.5)
                dk, dv = layer.dense()
                key = f"gate_d{dim}_t{length}_b{bits}"
                arrays[key] = _np(out)
                meta["gate"].append({
                    "key": key, "dim": dim, "length": length, "bits": bits, "seed": seed,
                    "inputs_sha": W.sha256(q, k, v), "dense_sha": W.sha256(dk, dv),
                    "page_bits": [pair[0].bits for pair in layer.pages],
                    "demotions": layer.demotions,
                    "payload_bytes": layer.payload_bytes,
                })

    p = W.PARITY
    mode_of = {16: CacheMode.FP16, 8: CacheMode.INT8, 4: CacheMode.INT4, 0: CacheMode.EVICTED}
    seed = 2026
    q, k, v, modes = W.parity_workload(seed)
    variants = {
        "global": dict(modes=modes, roles=None, directive=None),
        "evicted": dict(modes=W.draw_modes(seed + 4, len(modes),
                                           {16: 0.15, 8: 0.35, 4: 0.40, 0: 0.10}),
                        roles=None, directive=None),
        "focus": dict(modes=W.draw_modes(seed + 4, len(modes),
                                         {16: 0.15, 8: 0.35, 4: 0.40, 0: 0.10}),
                      roles="sink_scaffold_response", directive='<focus segments="5,9,20">'),
        "local": dict(modes=modes, roles="sink_scaffold_response", directive="<local>"),
    }
    scale = 1.0 / math.sqrt(p["dim"])
    for name, spec in variants.items():
        cache = DeclarativeKVCache(block_size=p["block"], group_size=p["group"])
        nblk = p["tokens"] // p["block"]
        roles = []
        for i in range(nblk):
            role = SegmentRole.CONTEXT
            if spec["roles"]:
                if i == 0:
                    role = SegmentRole.SINK
                elif i in (1, 2):
                    role = SegmentRole.SCAFFOLD
                elif i == nblk - 1:
                    role = SegmentRole.RESPONSE
            roles.append(role.value)
            sl = slice(i * p["block"], (i + 1) * p["block"])
            cache.add_segment(i, k[:, :, sl], v[:, :, sl], token_start=i * p["block"], role=role)
        for i, m in enumerate(spec["modes"]):
            if m != W.FP16:
                cache.requantize_segment(i, mode_of[m])
        if spec["directive"]:
            cache.feed_declarations(spec["directive"])
        visible = cache.visible_segment_ids()
        mat = cache.materialize_visible(dtype=torch.float16)
        g = p["q_heads"] // p["kv_heads"]
        out = F.scaled_dot_product_attention(q, mat.key.repeat_interleave(g, 1),
                                             mat.value.repeat_interleave(g, 1), scale=scale)
        key = f"parity_{name}"
        arrays[key] = _np(out)
        meta["parity"].append({
            "key": key, "seed": seed, "inputs_sha": W.sha256(q, k, v),
            "modes": [cache.segment_mode(i).value for i in range(nblk)],
            "roles": roles, "directive": spec["directive"], "visible": list(visible),
            "dense_sha": W.sha256(mat.key, mat.value), "tokens": int(mat.key.shape[-2]),
            "resident_bytes": cache.resident_bytes,
        })
    np.savez_compressed(HERE / "attention.npz", **arrays)
    (HERE / "attention.json").write_text(json.dumps(meta, indent=1))


def build_declarative(anchorkv):
    """The reference's DeclarativeKVCache on the page-format scenarios of
    workloads.DECLARATIVE: per recorded view the visible segments, positions,
    the storage report, sha256 digests of the dense K/V it materialises (in the
    original fp16 and as fp32 / bf16) and the SDPA output of every layer over
    the visible fp16 K/V."""
    from anchorkv.backend import DeclarativeKVCache, SegmentRole
    from anchorkv.policy import CacheMode

    arrays, meta = {}, []
    for spec in W.DECLARATIVE:
        kv, queries = W.declarative_inputs(spec)
        cache = DeclarativeKVCache(block_size=16, group_size=spec["group"])
        for sid, start, _, role in spec["segments"]:
            cache.add_segment(sid, kv[sid][0], kv[sid][1], token_start=start, role=SegmentRole(role))
        for step in spec["steps"]:
            if step[0] == "feed":
                cache.feed_declarations(step[1])
            else:
                cache.requantize_segment(step[1], CacheMode(step[2]))
        record = {"name": spec["name"], "inputs_sha": W.sha256(*[t for sid in sorted(kv) for t in kv[sid]],
                                                                 *queries), "views": []}
        for i, view in enumerate(spec["views"]):
            cache.feed_declarations(view)
            mat = cache.materialize_visible()
            f32 = cache.materialize_visible(dtype=torch.float32)
            b16 = cache.materialize_visible(dtype=torch.bfloat16)
            key5 = mat.key if mat.key.ndim == 5 else mat.key[None]
            val5 = mat.value if mat.value.ndim == 5 else mat.value[None]
            outs = []
            for layer, q in enumerate(queries):
                g = spec["q_heads"] // key5.shape[2]
                outs.append(F.scaled_dot_product_attention(
                    q, key5[layer].repeat_interleave(g, 1), val5[layer].repeat_interleave(g, 1),
                    scale=1.0 / math.sqrt(spec["dim"])))
            out_key = f"decl_{spec['name']}_{i}"
            arrays[out_key] = _np(torch.stack(outs))
            record["views"].append({
                "directive": view, "visible": list(cache.visible_segment_ids()),
                "positions": mat.positions.tolist(), "block_ids": list(mat.block_ids),
                "segment_ids": list(mat.segment_ids), "dense_sha_f16": W.sha256(mat.key, mat.value),
                "dense_sha_f32": W.sha256(f32.key, f32.value), "dense_sha_bf16": W.sha256(b16.key, b16.value),
                "shape": list(mat.key.shape), "report": cache.storage_report(), "out": out_key})
        meta.append(record)
    np.savez_compressed(HERE / "declarative.npz", **arrays)
    (HERE / "declarative.json").write_text(json.dumps(meta, indent=1))


def build_demo(anchorkv):
    from anchorkv.cli import run_requantization_demo
    from anchorkv.policy import CacheMode

    out = {m.value: run_requantization_demo(archive_mode=m) for m in (CacheMode.INT4, CacheMode.INT8)}
    (HERE / "demo.json").write_text(json.dumps(out, indent=1))


def main():
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_golden.py <reference source dir holding anchorkv/>")
    src = Path(sys.argv[1])
    sys.path.insert(0, str(src))
    import anchorkv

    torch.set_num_threads(max(1, torch.get_num_threads()))
    build_codec(anchorkv)
    build_attention(anchorkv)
    build_demo(anchorkv)
    build_declarative(anchorkv)
    print("wrote", sorted(p.name for p in HERE.iterdir() if p.suffix in (".npz", ".json")))


if __name__ == "__main__":
    main()
