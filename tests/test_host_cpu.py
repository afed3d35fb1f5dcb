"""Host-side logic that needs no GPU: checkpoint format and shape inference,
prompt assembly, attention split choice, frame byte accounting."""
import torch

from estudiocanciones_b200.checkpoint import (BASELINE_SHAPE, REFERENCE_SHAPE, TINY_SHAPE, linear_shapes,
                                              save_checkpoint, load_tensors, shape_from_tensors, synthetic_tensors)


def test_synthetic_checkpoint_roundtrip_and_shape(tmp_path):
    t = synthetic_tensors(TINY_SHAPE, seed=3)
    # reference key/dtype layout (app/convert_final.py:40-46)
    assert t["backbone.layers.0.attn.q_proj.weight.q8"].dtype == torch.int8
    assert t["backbone.layers.0.attn.q_proj.weight.s8"].dtype == torch.bfloat16
    assert t["audio_head.6.q8"].shape == (8197, TINY_SHAPE.dec_dim)
    assert t["unconditional_text_embedding.weight"].dtype == torch.bfloat16
    p = tmp_path / "m.safetensors"
    save_checkpoint(t, p)
    from safetensors import safe_open
    with safe_open(str(p), "pt") as f:
        assert f.metadata()["lite"] == '{"mode": "int8"}'
    t2 = load_tensors(p)
    assert all(torch.equal(t[k], t2[k]) for k in t)
    assert shape_from_tensors(t2, TINY_SHAPE.bb_heads, TINY_SHAPE.dec_heads) == TINY_SHAPE


def test_reference_and_baseline_shapes():
    assert REFERENCE_SHAPE.dec_hd == 384 and BASELINE_SHAPE.dec_hd == 128 and BASELINE_SHAPE.bb_hd == 128
    ls = linear_shapes(BASELINE_SHAPE)
    w = sum(n * k for key, (n, k) in ls.items() if key.startswith("backbone"))
    assert abs(w / 1e9 - 2.82) < 0.01          # backbone int8 bytes per frame
    assert ls["projection.weight"] == (1024, 3072)


def test_prompt_assembly_matches_reference_rules():
    from estudiocanciones_b200.engine import HeartMuLaLite

    class Tok:
        def encode(self, s):
            class R:
                pass
            r = R()
            r.ids = [ord(c) for c in s]
            return r
    ids, muq = HeartMuLaLite._prompt("Hola", "Pop, Rock", Tok())
    tags = "<tag>pop, rock</tag>"
    assert muq == len(tags) + 2
    assert ids[0] == 128000 and ids[muq - 1] == 128001 and ids[muq] == 0
    assert ids[muq + 1] == 128000 and ids[-1] == 128001
    assert bytes(ids[muq + 2:-1].tolist()).decode() == "hola"


def test_default_attention_split():
    from estudiocanciones_b200.engine import default_nsplit
    assert default_nsplit(8, 8, 1608, sms=148) == 4
    assert default_nsplit(1, 8, 768, sms=148) == 12
    assert default_nsplit(1, 8, 8192, sms=148) == 37
    assert default_nsplit(8, 2, 8, sms=148) == 1


def test_graph_capture_keeps_the_cyclic_collector_off():
    """Graph captures run with Python's cyclic collector off (a collection inside one could
    destroy a dead graph and invalidate the capture); its previous state comes back, also
    when the captured code raises."""
    import gc
    from estudiocanciones_b200._lib import capture_no_gc
    was = gc.isenabled()
    try:
        gc.enable()
        with capture_no_gc():
            assert not gc.isenabled()
        assert gc.isenabled()
        try:
            with capture_no_gc():
                raise RuntimeError("capture failed")
        except RuntimeError:
            pass
        assert gc.isenabled()
        gc.disable()
        with capture_no_gc():
            assert not gc.isenabled()
        assert not gc.isenabled()  # a caller that had it off keeps it off
    finally:
        (gc.enable if was else gc.disable)()


def test_stack_decode_plans_dropped_with_the_caches():
    """Stack.decode's per-shape launch plans hold raw pointers into the caches and weights:
    alloc() and free() (which the model's to() calls) drop them.  On the CPU, no launch."""
    from estudiocanciones_b200.engine import Linear, Stack
    t = synthetic_tensors(TINY_SHAPE, seed=5)

    def get(name, norm=False):
        return t[name].to(torch.float16) if norm else Linear(t[name + ".q8"], t[name + ".s8"])
    st = Stack(get, "backbone", TINY_SHAPE.bb_heads, t)
    st.alloc(2, 32, torch.device("cpu"))
    st._decode_plans["stale"] = object()
    st.alloc(2, 48, torch.device("cpu"))
    assert not st._decode_plans and st.L == 48
    st._decode_plans["stale"] = object()
    st.free()
    assert not st._decode_plans and st.blocks[0].kc is None
