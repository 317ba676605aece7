"""Operator-surface host logic on CPU: module construction and checkpoint
compatibility, exported names, argument checks, and no CPU fallback."""
import pytest
import torch

import modulated_deform_conv as mdc
import ms_deform_attn


def test_reference_exports_present():
    for name in ("ModulatedDeformConv2dFunction", "ModulatedDeformConv2d",
                 "ModulatedDeformConv2dPack", "modulated_deform_conv2d", "dcn_apply_nchw",
                 "dcn_split_nhwc", "gather_cols_nhwc", "DCNSplitNHWCFunction",
                 # modulated_deform_conv/__init__.py:2-10 of the reference
                 "ext_modulated_deformable_col2im_opt", "ext_modulated_deformable_col2im_smem",
                 "ext_modulated_deformable_col2im_coord_opt"):
        assert hasattr(mdc, name), name
    import msda_musa_opt2
    assert msda_musa_opt2.ms_deform_attn_forward is ms_deform_attn.ms_deform_attn_forward
    assert msda_musa_opt2.ms_deform_attn_backward is ms_deform_attn.ms_deform_attn_backward
    assert hasattr(ms_deform_attn, "MultiScaleDeformableAttnFunction")


def test_extension_exports_reference_op_names():
    import _modulated_deform_conv_ext as ext
    for name in ("modulated_deformable_im2col_cuda", "modulated_deformable_im2col_opt_cuda",
                 "modulated_deformable_im2col_nhwc_cuda", "dcn_forward", "dcn_pack_weight",
                 "modulated_deformable_fused_im2col_nhwc_cuda",
                 # backward ops, csrc/binding.cpp:146-191
                 "modulated_deformable_col2im_cuda", "modulated_deformable_col2im_opt_cuda",
                 "modulated_deformable_col2im_smem_cuda", "modulated_deformable_col2im_coord_cuda",
                 "modulated_deformable_col2im_coord_opt_cuda",
                 "modulated_deformable_col2im_nhwc_cuda",
                 "modulated_deformable_col2im_coord_nhwc_cuda",
                 "modulated_deformable_gradx_smem_nhwc_cuda",
                 "modulated_deformable_gradx_gather_nhwc_cuda",
                 "modulated_deformable_col2im_fused_smem_nhwc_cuda",
                 "modulated_deformable_col2im_perelem_nhwc_cuda",
                 "modulated_deformable_col2im_perelem_smem_nhwc_cuda"):
        assert hasattr(ext, name), name
    import _ms_deform_attn_ext as mext
    assert hasattr(mext, "forward") and hasattr(mext, "backward")


def test_module_parameters_match_mmcv_layout():
    m = mdc.ModulatedDeformConv2dPack(64, 32, 3, stride=1, padding=1, deform_groups=2,
                                      bias=False)
    sd = m.state_dict()
    assert set(sd) == {"weight", "conv_offset.weight", "conv_offset.bias"}
    assert sd["weight"].shape == (32, 64, 3, 3)
    assert sd["conv_offset.weight"].shape == (2 * 3 * 9, 64, 3, 3)
    assert torch.count_nonzero(sd["conv_offset.weight"]) == 0      # zero-initialised offsets
    m2 = mdc.ModulatedDeformConv2d(16, 8, (3, 1), groups=2)
    assert m2.weight.shape == (8, 8, 3, 1) and m2.bias.shape == (8,)
    assert float(m2.weight.detach().abs().max()) <= 1.0 / (16 * 3) ** 0.5 + 1e-7


def test_state_dict_v1_offset_key_migration():
    """Version-1 checkpoints name the offset conv "<prefix>_offset"; loading renames
    the keys to conv_offset (modulated_deform_conv.py:629-643).  Torch filters the
    state dict per child prefix, so the rename applies where the module is the root
    of the load, exactly as in the reference."""
    m = mdc.ModulatedDeformConv2dPack(8, 8, 3, padding=1)
    sd = {k: v.clone() for k, v in m.state_dict().items()}
    w = torch.randn_like(sd["conv_offset.weight"])
    b = torch.randn_like(sd["conv_offset.bias"])
    old = torch.nn.modules.module.OrderedDict(
        [("weight", sd["weight"]), ("bias", sd["bias"]), ("_offset.weight", w),
         ("_offset.bias", b)])
    old._metadata = {"": {"version": 1}}
    m.load_state_dict(old)
    assert torch.equal(m.conv_offset.weight, w) and torch.equal(m.conv_offset.bias, b)


def test_backend_kwarg_accepted(monkeypatch):
    monkeypatch.setenv("DCN_BACKEND", "tilelang")
    m = mdc.ModulatedDeformConv2dPack(8, 8, 3, padding=1, backend="cuda")
    assert m.backend == "cuda"
    m2 = mdc.ModulatedDeformConv2dPack(8, 8, 3, padding=1)
    assert m2.backend == "tilelang"


def test_no_cpu_fallback():
    x = torch.randn(1, 8, 6, 6)
    off = torch.zeros(1, 18, 6, 6)
    mask = torch.ones(1, 9, 6, 6)
    w = torch.randn(8, 8, 3, 3)
    with pytest.raises(RuntimeError, match="CUDA"):
        mdc.modulated_deform_conv2d(x, off, mask, w, None, 1, 1, 1)
    with pytest.raises(RuntimeError, match="CUDA"):
        ms_deform_attn.ms_deform_attn_forward(torch.randn(1, 4, 1, 32),
                                              torch.tensor([[2, 2]]), torch.tensor([0]),
                                              torch.rand(1, 3, 1, 1, 1, 2),
                                              torch.rand(1, 3, 1, 1, 1))


def test_function_rejects_non_4d_input():
    with pytest.raises(ValueError):
        mdc.modulated_deform_conv2d(torch.randn(8, 6, 6), torch.zeros(1), torch.zeros(1),
                                    torch.zeros(1, 8, 3, 3))


def test_sharding_blocks_cover_exactly():
    from bevk.sharding import shard_range
    for n in (48, 7, 1, 0):
        for world in (1, 2, 4, 8):
            blocks = [shard_range(n, r, world) for r in range(world)]
            assert blocks[0][0] == 0 and blocks[-1][1] == n
            assert all(b[1] == c[0] for b, c in zip(blocks, blocks[1:]))
            sizes = [e - b for b, e in blocks]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


class _FakePackExt:
    """Stands in for the extension's packing op on the CPU: counts the calls
    and returns a copy, so a test sees when the cache is (not) used."""

    def __init__(self):
        self.calls = 0

    def dcn_pack_weight(self, w, groups):
        self.calls += 1
        return w.clone()


def test_weight_caches_follow_data_swaps(monkeypatch):
    """The derived-weight caches see `p.data = t` (new storage, old version
    counter) and optimizer-style in-place updates; `p.data.copy_(t)` is
    invisible to them until invalidate_weight_caches."""
    from modulated_deform_conv import modulated_deform_conv as impl
    fake = _FakePackExt()
    monkeypatch.setattr(impl, "_load_ext", lambda: fake)
    p = torch.nn.Parameter(torch.randn(8, 4, 3, 3))
    a = impl.packed_weight(p)
    assert impl.packed_weight(p) is a and fake.calls == 1          # cached
    new = torch.randn(8, 4, 3, 3)
    p.data = new                                                   # EMA / loader swap
    b = impl.packed_weight(p)
    assert fake.calls == 2 and torch.equal(b, new)
    before = new.clone()
    with torch.no_grad():
        p.mul_(2.0)                                                # optimizer-style update
    c = impl.packed_weight(p)
    assert fake.calls == 3 and torch.equal(c, 2.0 * before)
    p.data.copy_(torch.zeros(8, 4, 3, 3))                          # not visible to the key
    assert impl.packed_weight(p) is c
    impl.invalidate_weight_caches(p)
    assert torch.equal(impl.packed_weight(p), torch.zeros(8, 4, 3, 3)) and fake.calls == 4


def test_tap_major_and_bn_fold_caches_follow_data_swaps():
    from modulated_deform_conv import modulated_deform_conv as impl
    from modulated_deform_conv.dcn_split_nhwc import _fold_bn
    w = torch.nn.Parameter(torch.randn(6, 4, 3, 3))
    t1 = impl._tap_major_weight(w, torch.float32)
    w.data = torch.randn(6, 4, 3, 3)
    t2 = impl._tap_major_weight(w, torch.float32)
    assert torch.equal(t2, w.detach().permute(0, 2, 3, 1).reshape(6, 36))
    assert not torch.equal(t1, t2)
    scale, shift = torch.rand(6) + 0.5, torch.randn(6)
    w1, _ = _fold_bn(w, None, scale, shift)
    scale.data = torch.rand(6) + 2.0                                  # swapped BN buffer
    w2, _ = _fold_bn(w, None, scale, shift)
    assert torch.allclose(w2, w.detach() * scale.view(-1, 1, 1, 1))
    assert not torch.equal(w1, w2)
    # module-wide invalidation clears every cached copy on its tensors
    m = impl.ModulatedDeformConv2d(4, 6, 3, padding=1)
    impl._tap_major_weight(m.weight, torch.float32)
    assert hasattr(m.weight, "_bevk_tap_major")
    impl.invalidate_weight_caches(m)
    assert not hasattr(m.weight, "_bevk_tap_major")
