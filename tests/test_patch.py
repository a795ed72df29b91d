"""The runtime patch (deepseek_v4_kernel._patch) on CPU, with stand-in
modules for flash_mla and SGLang (neither is installed here).

* flash_mla_with_kvcache is replaced by a wrapper; calls that do not take
  the B200 path (here: no sm_100 device) reach the original unchanged, and
  patching is idempotent (reference deepseek_v4_kernel/_patch.py:161-197).
* SGLang's two indexer fallbacks get a [b, 1] seq_lens squeezed to [b]
  (reference _patch.py:199-236); other arguments pass through.
"""
import sys
import types

import pytest
import torch


@pytest.fixture
def fake_modules(monkeypatch):
    calls = []

    def flash_mla_with_kvcache(*args, **kwargs):
        calls.append(("flash_mla", args, kwargs))
        return "upstream"

    fmi = types.ModuleType("flash_mla.flash_mla_interface")
    fmi.flash_mla_with_kvcache = flash_mla_with_kvcache
    fmi.FlashMLASchedMeta = type("FlashMLASchedMeta", (), {})
    pkg = types.ModuleType("flash_mla")
    pkg.flash_mla_interface = fmi
    pkg.flash_mla_with_kvcache = flash_mla_with_kvcache

    def strict_1d(q_fp8, kvcache_fp8, weight, seq_lens, *args, **kwargs):
        assert seq_lens.dim() == 1, "fallback asserts 1-D seq_lens"
        calls.append(("indexer", seq_lens.tolist(), args, kwargs))
        return seq_lens.sum().item()

    tk = types.ModuleType("sglang.srt.layers.attention.nsa.tilelang_kernel")
    tk.tilelang_fp8_paged_mqa_logits = strict_1d
    idx = types.ModuleType("sglang.srt.layers.attention.compressed.indexer")
    idx.fp8_paged_mqa_logits_torch = strict_1d
    for name, mod in {"flash_mla": pkg, "flash_mla.flash_mla_interface": fmi,
                      "sglang.srt.layers.attention.nsa.tilelang_kernel": tk,
                      "sglang.srt.layers.attention.compressed.indexer": idx}.items():
        monkeypatch.setitem(sys.modules, name, mod)
    from deepseek_v4_kernel import _patch
    monkeypatch.setattr(_patch, "_INSTALLED", False)
    return calls, pkg, fmi, tk, idx


def test_install_wraps_and_defers_off_device(fake_modules):
    from deepseek_v4_kernel import _patch
    calls, pkg, fmi, tk, idx = fake_modules
    assert _patch.install()
    assert getattr(fmi.flash_mla_with_kvcache, "__dsv4b_patched__", False)
    assert pkg.flash_mla_with_kvcache is fmi.flash_mla_with_kvcache
    q = torch.zeros(1, 1, 16, 576, dtype=torch.bfloat16)
    kv = torch.zeros(1, 64, 1, 656, dtype=torch.uint8)
    out = fmi.flash_mla_with_kvcache(q, kv, None, None, 512, None, is_fp8_kvcache=True,
                                     indices=torch.zeros(1, 1, 64, dtype=torch.int32))
    assert out == "upstream" and calls[-1][0] == "flash_mla"   # CPU tensors: not the B200 path
    wrapped = fmi.flash_mla_with_kvcache
    _patch._INSTALLED = False
    _patch.install()                                            # idempotent
    assert fmi.flash_mla_with_kvcache is wrapped


def test_indexer_fallbacks_get_1d_seq_lens(fake_modules):
    from deepseek_v4_kernel import _patch
    calls, _, _, tk, idx = fake_modules
    assert _patch._patch_sglang_indexer_fallbacks() == 2
    for fn in (tk.tilelang_fp8_paged_mqa_logits, idx.fp8_paged_mqa_logits_torch):
        assert fn(None, None, None, torch.tensor([[3], [4]]), 7, clean=True) == 7
        assert calls[-1] == ("indexer", [3, 4], (7,), {"clean": True})
        assert fn(None, None, None, torch.tensor([5, 6])) == 11              # 1-D untouched
        with pytest.raises(AssertionError):
            fn(None, None, None, torch.tensor([[1, 2]]))                    # [1, 2] is not squeezed
    first = tk.tilelang_fp8_paged_mqa_logits
    assert _patch._patch_sglang_indexer_fallbacks() == 2
    assert tk.tilelang_fp8_paged_mqa_logits is first                      # idempotent


def test_disable_env(fake_modules, monkeypatch):
    from deepseek_v4_kernel import _patch
    monkeypatch.setenv("DSV4B_KERNEL_DISABLE", "1")
    assert not _patch.install()
