"""The vLLM attention backend's host logic, without a GPU or a vLLM engine.

Mirrors the behaviour of the reference backend (glm53_sparse_mla/backend.py of
the reference): capability / dtype / head-size gates, the kv-cache shape, the
metadata builder reporting every token as a decode token, the impl's argument
checks, and the env-gated registration. The reference ships no test for its
backend; forward_mqa itself needs a GPU (tests/test_backend_gpu.py).
"""

from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

pytest.importorskip("vllm")

from glm53_sparse_mla import backend as B  # noqa: E402
from vllm.platforms.interface import DeviceCapability  # noqa: E402
from vllm.v1.attention.backend import AttentionCGSupport  # noqa: E402


def test_backend_class_api():
    be = B.Glm53SparseMLABackend
    assert be.get_name() == "FLASHINFER_MLA_SPARSE"
    assert be.get_supported_head_sizes() == [512]
    assert be.get_kv_cache_shape(10, 64, 1, 512) == (10, 64, 512)
    assert be.is_mla() and be.is_sparse()
    assert "fp8" in be.supported_kv_cache_dtypes and "bfloat16" in be.supported_kv_cache_dtypes
    assert be.get_impl_cls() is B.Glm53SparseMLAImpl
    assert be.get_builder_cls() is B.Glm53SparseMLAMetadataBuilder
    assert be.get_metadata_cls() is B.Glm53SparseMLAMetadata


def test_capability_gate_is_sm100():
    be = B.Glm53SparseMLABackend
    assert be.supports_compute_capability(DeviceCapability(10, 0))
    assert not be.supports_compute_capability(DeviceCapability(12, 0))
    assert not be.supports_compute_capability(DeviceCapability(9, 0))


def test_supports_combination():
    f = B.Glm53SparseMLABackend.supports_combination
    cap = DeviceCapability(10, 0)
    ok = dict(head_size=512, dtype=torch.bfloat16, kv_cache_dtype="auto", block_size=64,
              use_mla=True, has_sink=False, use_sparse=True, use_mm_prefix=False,
              device_capability=cap)
    assert f(**ok) is None
    assert "sparse" in f(**{**ok, "use_sparse": False})
    assert "NoPE" in f(**{**ok, "head_size": 576})
    assert "sink" in f(**{**ok, "has_sink": True})


def test_builder_reports_all_tokens_as_decode():
    assert B.Glm53SparseMLAMetadataBuilder._cudagraph_support == AttentionCGSupport.UNIFORM_BATCH
    cfg = SimpleNamespace(model_config=SimpleNamespace(hf_config=SimpleNamespace(index_topk=2048)),
                          scheduler_config=SimpleNamespace(max_num_batched_tokens=64))
    spec = SimpleNamespace(block_size=64)
    b = B.Glm53SparseMLAMetadataBuilder(spec, ["l0"], cfg, torch.device("cpu"))
    qsl = torch.tensor([0, 3, 4, 9], dtype=torch.int32)
    cm = SimpleNamespace(num_actual_tokens=9, query_start_loc=qsl, query_start_loc_cpu=qsl,
                         num_reqs=3, max_query_len=5, max_seq_len=100,
                         slot_mapping=torch.zeros(9, dtype=torch.int64),
                         block_table_tensor=torch.zeros(3, 4, dtype=torch.int32))
    md = b.build(0, cm)
    assert md.req_id_per_token.tolist() == [0, 0, 0, 1, 2, 2, 2, 2, 2]
    assert md.num_decode_tokens == 9 and md.num_prefills == 0 and md.num_decodes == 3
    assert md.topk_tokens == 2048 and md.block_size == 64
    # the persistent buffer is reused (stable storage for graph capture)
    assert md.req_id_per_token.data_ptr() == b.req_id_per_token_buffer.data_ptr()


def _impl(**kw):
    args = dict(num_heads=64, head_size=512, scale=512 ** -0.5, num_kv_heads=1, alibi_slopes=None,
                sliding_window=None, kv_cache_dtype="auto", logits_soft_cap=None,
                attn_type="decoder", kv_sharing_target_layer_name=None,
                topk_indices_buffer=torch.zeros(4, 2048, dtype=torch.int32), kv_lora_rank=512)
    args.update(kw)
    return B.Glm53SparseMLAImpl(**args)


def test_impl_argument_checks():
    impl = _impl()
    assert impl.kv_lora_rank == 512 and impl.softmax_scale == 512 ** -0.5
    for h in (8, 16, 32, 64):
        _impl(num_heads=h)
    with pytest.raises(NotImplementedError):
        _impl(num_heads=12)
    with pytest.raises(NotImplementedError):
        _impl(sliding_window=128)
    with pytest.raises(NotImplementedError):
        _impl(kv_cache_dtype="fp8_ds_mla").forward_mqa(
            torch.zeros(1, 64, 512), torch.zeros(1, 64, 512), None, None)
    # an indexer's buffer takes precedence over the explicit one
    buf = torch.ones(2, 2, dtype=torch.int32)
    assert _impl(indexer=SimpleNamespace(topk_indices_buffer=buf)).topk_indices_buffer is buf


def test_kv_scale_lookup():
    kv8 = torch.zeros(4, 512, dtype=torch.float8_e4m3fn)
    kvb = torch.zeros(4, 512, dtype=torch.bfloat16)
    f = B.Glm53SparseMLAImpl._kv_scale
    assert f(SimpleNamespace(_k_scale_float=0.25), kvb) == 1.0
    assert f(SimpleNamespace(_k_scale_float=0.25), kv8) == 0.25
    assert f(SimpleNamespace(_k_scale=torch.tensor(0.5)), kv8) == 0.5
    assert f(SimpleNamespace(), kv8) == 1.0


def test_register_is_env_gated(monkeypatch):
    from vllm.v1.attention.backends import registry as R
    monkeypatch.delenv("VLLM_GLM53_CUDA_SPARSE_MLA", raising=False)
    assert B.register() is False
    monkeypatch.setenv("VLLM_GLM53_CUDA_SPARSE_MLA", "1")
    saved = dict(R._ATTN_OVERRIDES)
    try:
        assert B.register() is True
        slot = R.AttentionBackendEnum.FLASHINFER_MLA_SPARSE
        assert R._ATTN_OVERRIDES[slot] == "glm53_sparse_mla.backend.Glm53SparseMLABackend"
        monkeypatch.setenv("VLLM_GLM53_BACKEND_SLOT", "NO_SUCH_SLOT")
        with pytest.raises(ValueError):
            B.register()
    finally:
        R._ATTN_OVERRIDES.clear()
        R._ATTN_OVERRIDES.update(saved)
