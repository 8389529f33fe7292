"""Inference plugins (reference teco/plugin/plugin*/plugin_*.cc) driven through the
stand-in plugin host: registration and InferOutputShape need no GPU."""
from tecoops import plugin


def test_plugins_registered_with_reference_inputs():
    reg = plugin.registered()
    assert reg["plugin_reshape_and_cache"] == ["key", "value", "slot_mapping"]
    assert reg["plugin_flash_attention"] == ["q", "k_cache", "v_cache", "block_table",
                                             "cu_seqlens_q", "seqused_k"]


def test_reshape_plugin_output_shape():
    # plugin_reshape_and_cache.cc:56-60: [2 * num_blocks, H, block_size, D]
    shape = plugin.infer_output_shape("plugin_reshape_and_cache",
                                      [[512, 8, 128], [512, 8, 128], [512]],
                                      {"num_blocks": 64, "block_size": 16})
    assert shape == [128, 8, 16, 128]


def test_flash_plugin_output_shape_is_q_shape():
    shape = plugin.infer_output_shape(
        "plugin_flash_attention",
        [[385, 32, 128], [256, 8, 32, 128], [256, 8, 32, 128], [3, 16], [4], [3]],
        {"max_seqlen_q": 512, "max_seqlen_k": 1024, "max_block_num": 256})
    assert shape == [385, 32, 128]


def test_unknown_plugin_and_missing_attribute():
    import pytest
    with pytest.raises(RuntimeError):
        plugin.infer_output_shape("plugin_nope", [[1]], {})
    with pytest.raises(RuntimeError):
        plugin.infer_output_shape("plugin_reshape_and_cache", [[4, 2, 8], [4, 2, 8], [4]],
                                  {"num_blocks": 4})


def test_rms_norm_plugins_registered_and_shapes():
    """plugin_rms_norm / plugin_rms_norm_add (reference
    teco/plugin/pluginRmsNorm/plugin_rms_norm.cc): outputs shaped like the input."""
    reg = plugin.registered()
    assert reg["plugin_rms_norm"] == ["input", "weight"]
    assert reg["plugin_rms_norm_add"] == ["input", "weight", "residual"]
    assert plugin.infer_output_shape("plugin_rms_norm", [[64, 4096], [4096]],
                                     {"eps": 1e-6}) == [64, 4096]
    assert plugin.infer_output_shape("plugin_rms_norm_add", [[7, 128], [128], [7, 128]],
                                     {"eps": 1e-5}, n_out=2) == [[7, 128], [7, 128]]
