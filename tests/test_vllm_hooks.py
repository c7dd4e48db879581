"""vLLM-Omni plugin glue on CPU (mirrors the reference plugin's
test_register / test_*_hook / test_fallback_warnings / step-tracker
behaviour): env-gated installers, deferred vllm-omni imports, the shared hook
state's step counting and pattern cache, the mask-log selector, fallback
warnings."""

import importlib
import os

import pytest
import torch


@pytest.fixture(autouse=True)
def clean_env(monkeypatch):
    for key in list(os.environ):
        if key.startswith("LVSA_"):
            monkeypatch.delenv(key, raising=False)
    yield


def test_register_surface_and_lazy_imports():
    from longvideosparseattention_b200.vllm_omni import register
    for f in ("register_lvsa_backend", "maybe_install_hunyuan_hook", "maybe_install_wan_hook",
              "maybe_install_cosmos3_hook"):
        assert hasattr(register, f)
    with pytest.raises((ImportError, ModuleNotFoundError)):
        register.register_lvsa_backend()


@pytest.mark.parametrize("env,fn", [("LVSA_HUNYUAN_HOOK", "maybe_install_hunyuan_hook"),
                                    ("LVSA_WAN_HOOK", "maybe_install_wan_hook"),
                                    ("LVSA_COSMOS3_HOOK", "maybe_install_cosmos3_hook")])
def test_env_gated_installers(env, fn, monkeypatch, capsys):
    from longvideosparseattention_b200.vllm_omni import register
    getattr(register, fn)()                     # disabled: silent
    assert capsys.readouterr().out == ""
    monkeypatch.setenv(env, "0")
    getattr(register, fn)()
    assert capsys.readouterr().out == ""
    monkeypatch.setenv(env, "1")
    getattr(register, fn)()                     # no T_lat: warning
    assert "Warning" in capsys.readouterr().out
    monkeypatch.setenv("LVSA_TOTAL_LATENT_FRAMES", "33")
    getattr(register, fn)()                     # vllm-omni absent: reported, not raised
    assert "failed" in capsys.readouterr().out


@pytest.mark.parametrize("mod,fn", [("hunyuan_hook", "install_hunyuan_lvsa_hook"),
                                    ("wan_hook", "install_wan_lvsa_hook"),
                                    ("cosmos3_hook", "install_cosmos3_lvsa_hook")])
def test_install_needs_vllm_omni(mod, fn):
    m = importlib.import_module(f"longvideosparseattention_b200.vllm_omni.{mod}")
    with pytest.raises((ImportError, ModuleNotFoundError)):
        getattr(m, fn)(total_latent_frames=21)


def test_hooks_share_the_state_class():
    from longvideosparseattention_b200.vllm_omni import cosmos3_hook, hunyuan_hook, wan_hook
    assert wan_hook.HunyuanLVSAState is hunyuan_hook.HunyuanLVSAState
    assert cosmos3_hook.HunyuanLVSAState is hunyuan_hook.HunyuanLVSAState


def test_mask_log_selector():
    from longvideosparseattention_b200.vllm_omni.hunyuan_hook import _mask_log_should_fire as f
    assert not f("", 0, -1) and not f("0", 10, 3)
    assert f("1", 0, -1) and f("1", 1, 0) and not f("1", 5, 5)
    assert f("once", 0, -1) and not f("once", 1, 0)
    assert f("3-7", 3, -1) and f("3-7", 7, -1) and not f("3-7", 2, -1) and not f("3-7", 8, -1)
    assert f("2,5,10", 5, -1) and not f("2,5,10", 3, -1)
    assert f("abc", 0, -1) is False and f("3-abc", 5, -1) is False


def test_state_tick(monkeypatch):
    from longvideosparseattention_b200.vllm_omni.config import LVSAConfig
    from longvideosparseattention_b200.vllm_omni.hunyuan_hook import HunyuanLVSAState
    s = HunyuanLVSAState(LVSAConfig())
    assert s.tick(layer_id=1, seq_len=100) == 0
    s.tick(layer_id=2, seq_len=100)
    s.tick(layer_id=1, seq_len=200)           # new sequence length: new generation
    assert s._generation_seq_len == 200 and s._step == 0
    monkeypatch.setenv("LVSA_CFG_PASSES", "1")
    s = HunyuanLVSAState(LVSAConfig())
    for lid in (1, 2, 3):
        s.tick(layer_id=lid, seq_len=100)
    assert s._n_blocks is None
    s.tick(layer_id=1, seq_len=100)           # first repeat calibrates n_blocks
    assert s._n_blocks == 3 and s._step == 1
    for lid in (2, 3, 1):
        s.tick(layer_id=lid, seq_len=100)
    assert s._step == 2


def test_state_metadata_cache():
    from longvideosparseattention_b200.vllm_omni.config import LVSAConfig
    from longvideosparseattention_b200.vllm_omni.hunyuan_hook import HunyuanLVSAState
    cpu = torch.device("cpu")
    s = HunyuanLVSAState(LVSAConfig(rotate_keyframes=False))
    m1 = s.get_metadata(33, 1560, 0, cpu)
    assert s.get_metadata(33, 1560, 5, cpu) is m1          # no rotation: cached across steps
    assert s.get_metadata(49, 1560, 0, cpu) is not m1 and s._cached_total_frames == 49
    s = HunyuanLVSAState(LVSAConfig(rotate_keyframes=True, reference_latent_frames=12))
    assert s.get_metadata(49, 1560, 0, cpu) is not s.get_metadata(49, 1560, 1, cpu)
    # Cosmos3-Nano geometry: dense at the native horizon (48), sparse at 2x.
    s = HunyuanLVSAState(LVSAConfig(reference_latent_frames=48))
    m = s.get_metadata(48, 920, 0, cpu)
    assert m.key_frame_interval == 1 and len(m.global_indices) == 48
    m = s.get_metadata(96, 920, 0, cpu)
    assert len(m.global_indices) < 96


@pytest.fixture
def fallback(monkeypatch):
    monkeypatch.setenv("LVSA_WARN_FALLBACK", "1")
    import longvideosparseattention_b200.vllm_omni._fallback as fb
    importlib.reload(fb)
    fb.reset_warnings()
    yield fb
    fb.reset_warnings()


def test_fallback_warnings(fallback, capsys, monkeypatch):
    fallback.warn_fallback("origin_a", "reason_x", 100, {"k": "v"})
    out = capsys.readouterr().out
    assert "[LVSA-FALLBACK]" in out and "origin_a" in out and "reason_x" in out
    assert "seq_len=100" in out and "k=v" in out
    fallback.warn_fallback("origin_a", "reason_x", 100)
    assert capsys.readouterr().out == ""                   # deduplicated
    fallback.warn_fallback("origin_a", "reason_x", 101)
    fallback.warn_fallback("origin_a", "reason_y", 101)
    out = capsys.readouterr().out
    assert out.count("origin_a") == 2
    fallback.reset_warnings()
    fallback.warn_fallback("origin_a", "reason_x", 100)
    assert "origin_a" in capsys.readouterr().out
    monkeypatch.setenv("LVSA_WARN_FALLBACK", "0")
    importlib.reload(fallback)
    fallback.warn_fallback("origin_b", "reason_x", 100)
    assert capsys.readouterr().out == ""


def test_block_count_step_tracker():
    from longvideosparseattention_b200.vllm_omni import step_tracker as st
    st.reset()
    t = st.BlockCountStepTracker()
    assert [t.tick() for _ in range(3)] == [0, 0, 0]
    t.mark_step_boundary()                   # first step had 3 blocks
    assert t.n_blocks == 3 and t.current_step == 1
    assert [t.tick() for _ in range(4)] == [1, 1, 1, 2]
    assert st.get_step() == 2
    t2 = st.BlockCountStepTracker()
    t2.set_n_blocks(2)
    assert [t2.tick() for _ in range(5)] == [0, 0, 1, 1, 2]
    st.set_total_latent_frames(21)
    st.set_num_patches(1560)
    assert st.get_total_latent_frames() == 21 and st.get_num_patches() == 1560
    assert st.tick_self_attention() == 0
    st.reset()
    assert st.get_total_latent_frames() is None and st.get_step() == 0
