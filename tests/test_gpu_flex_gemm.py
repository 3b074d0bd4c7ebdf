"""The drop-in flex_gemm package on the GPU: caches bit-exact against the reference's own fixtures (neighbour maps,
pooled coordinates, parent / seg_indices / seg_offsets), pooling and upsampling bit-exact against the reference
formulas, the float conv against an fp32/fp64 torch restatement of the reference operator, and a ResBlock + PoolDown +
NearestUp chain built from the nn modules the way the refiner's blocks call them."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

SMALL = ["B_small", "A_small"]


def _widths(g):
    from promptmoge_b200 import synth
    return synth.MODELS[g.config["model"]]["model_channels"]


def _level_shapes(g, L):
    shape = [int(s) for s in g["s0_shape"]]
    out = [tuple(shape)]
    for _ in range(L - 1):
        b, h, w, z = out[-1]
        out.append((b, -(-h // 2), -(-w // 2), -(-z // 2)))
    return out


@pytest.mark.parametrize("name", SMALL)
def test_caches_match_reference_fixtures(golden, name):
    from promptmoge_b200.flex_gemm.ops import build_pool_cache, build_submanifold_cache
    g = golden(name)
    L = len(_widths(g))
    shapes = _level_shapes(g, L)
    for k in range(L):
        coords = torch.from_numpy(g[f"s0_L{k}_coords"]).cuda()
        cache = build_submanifold_cache(coords, shapes[k], (3, 3, 3))
        np.testing.assert_array_equal(cache.nmap.cpu().numpy(), g[f"s0_L{k}_nmap"], err_msg=f"L{k} nmap")
        assert cache.num_input_coords == cache.num_output_coords == coords.shape[0]
        if k + 1 < L:
            pc = build_pool_cache(coords, shapes[k], (2, 2, 2), (2, 2, 2), (0, 0, 0))
            np.testing.assert_array_equal(pc.output_coords.cpu().numpy(), g[f"s0_L{k + 1}_coords"], err_msg=f"P{k}")
            for key in ("parent", "seg_indices", "seg_offsets"):
                ref = g[f"s0_P{k}_{key}"]
                got = getattr(pc, key).cpu().numpy()
                assert got.dtype == ref.dtype, (key, got.dtype, ref.dtype)
                np.testing.assert_array_equal(got, ref, err_msg=f"P{k} {key}")
            assert tuple(pc.output_sparse_shape) == shapes[k + 1]
            assert pc.T.is_transposed and pc.T.T is pc


def _torch_conv(x, nmap, w, b):
    """The reference operator (_core.py:399-441) in float64 on the CPU."""
    M, Co = x.shape[0], w.shape[0]
    wv = w.reshape(Co, 27, -1).double()
    out = b.double().repeat(M, 1)
    for v in range(27):
        rows = torch.nonzero(nmap[:, v] >= 0).flatten()
        out.index_add_(0, rows, x.double()[nmap[rows, v].long()] @ wv[:, v, :].t())
    return out


@pytest.mark.parametrize("name", SMALL)
def test_functional_ops_against_reference_formulas(golden, name):
    from promptmoge_b200.flex_gemm.ops import (build_pool_cache, sparse_pool, sparse_upsample, submanifold_conv)
    g = golden(name)
    L = len(_widths(g))
    shapes = _level_shapes(g, L)
    gen = torch.Generator().manual_seed(3)
    with torch.no_grad():
        for k in range(2):
            coords = torch.from_numpy(g[f"s0_L{k}_coords"]).cuda()
            M, C = coords.shape[0], 16 * (k + 2)
            x = torch.randn((M, C), generator=gen)
            w = torch.randn((24, 3, 3, 3, C), generator=gen) * 0.05
            b = torch.randn(24, generator=gen)
            out, cache = submanifold_conv(x.cuda(), coords, torch.Size([*shapes[k], C]), w.cuda(), b.cuda())
            want = _torch_conv(x, torch.from_numpy(g[f"s0_L{k}_nmap"]), w, b)
            np.testing.assert_allclose(out.cpu().numpy(), want.numpy(), rtol=1e-4, atol=1e-4)
            # the cache is reused (no rebuild) and a stale one is refused
            out2, cache2 = submanifold_conv(x.cuda(), coords, torch.Size([*shapes[k], C]), w.cuda(), b.cuda(),
                                            neighbor_cache=cache)
            assert cache2 is cache and torch.equal(out2, out)
            # pooling: children summed in ascending fine index in fp32, then / count (index_add_ + bincount)
            pc = build_pool_cache(coords, shapes[k], (2, 2, 2), (2, 2, 2), (0, 0, 0))
            pooled, pcoords, pshape, _ = sparse_pool(x.cuda(), coords, torch.Size([*shapes[k], C]), (2, 2, 2),
                                                     neighbor_cache=pc)
            parent = pc.parent.cpu().long()
            acc = torch.zeros((pcoords.shape[0], C))
            acc.index_add_(0, parent, x)
            cnt = torch.bincount(parent, minlength=pcoords.shape[0]).clamp(min=1).float()
            assert torch.equal(pooled.cpu(), acc / cnt[:, None])
            summed, _, _, _ = sparse_pool(x.cuda(), coords, torch.Size([*shapes[k], C]), (2, 2, 2), reduce="sum",
                                          neighbor_cache=pc)
            assert torch.equal(summed.cpu(), acc)
            assert tuple(pshape) == (*shapes[k + 1], C)
            up, ucoords, ushape, _ = sparse_upsample(pooled, pcoords, pshape, (2, 2, 2), output_coords=coords,
                                                     output_shape=torch.Size([*shapes[k], C]),
                                                     neighbor_cache=pc.T)
            assert torch.equal(up.cpu(), pooled.cpu()[parent]) and ucoords is coords


def test_resblock_pool_up_chain_matches_torch_reference(golden):
    """SparseResBlock3d + PoolDown + NearestUp (flex_sparse_blocks.py:50-105) built on the drop-in nn modules, against
    the same chain written with the reference operator formulas in float64 torch on the CPU."""
    from promptmoge_b200.flex_gemm import nn as fnn
    g = golden("A_small")
    shapes = _level_shapes(g, 5)
    coords = torch.from_numpy(g["s0_L0_coords"]).cuda()
    C = 32
    torch.manual_seed(5)
    norm = torch.nn.LayerNorm(C, eps=1e-6)
    conv1, conv2 = fnn.SubmanifoldConv3d(C, C, 3), fnn.SubmanifoldConv3d(C, C, 3)
    pool = fnn.SparsePool3d(kernel_size=2, stride=2, reduce="mean")
    up = fnn.SparseUpsample3d(scale_factor=2, mode="nearest")
    lin = torch.nn.Linear(C, C)
    x = torch.randn(coords.shape[0], C)
    shape = torch.Size([*shapes[0], C])
    with torch.no_grad():
        h = torch.nn.functional.silu(norm(x))
        h, cache = conv1.cuda()(h.cuda(), coords, shape)
        h = torch.nn.functional.silu(h)
        h, cache = conv2.cuda()(h, coords, shape, neighbor_cache=cache)
        y = h + x.cuda()
        p, pc_coords, pshape, down = pool(y, coords, shape, output_shape=torch.Size([*shapes[1], C]))
        p = lin.cuda()(p)
        u, _, _, _ = up(p, pc_coords, pshape, output_coords=coords, output_shape=shape, neighbor_cache=down.T)
        got = (u + y).cpu()
        nm = torch.from_numpy(g["s0_L0_nmap"])
        h = torch.nn.functional.silu(norm.cpu()(x)).double()
        h = _torch_conv(h, nm, conv1.weight.cpu(), conv1.bias.cpu())
        h = _torch_conv(torch.nn.functional.silu(h), nm, conv2.weight.cpu(), conv2.bias.cpu())
        yr = h + x.double()
        parent = torch.from_numpy(g["s0_P0_parent"]).long()
        acc = torch.zeros((int(parent.max()) + 1, C), dtype=torch.float64).index_add_(0, parent, yr)
        acc = acc / torch.bincount(parent).double()[:, None]
        pr = acc @ lin.weight.cpu().double().t() + lin.bias.cpu().double()
        want = pr[parent] + yr
    np.testing.assert_allclose(got.numpy(), want.numpy(), rtol=1e-3, atol=1e-3)


def test_gradients_are_refused(golden):
    from promptmoge_b200.flex_gemm import nn as fnn
    g = golden("B_small")
    coords = torch.from_numpy(g["s0_L1_coords"]).cuda()
    conv = fnn.SubmanifoldConv3d(8, 8, 3).cuda()
    x = torch.randn(coords.shape[0], 8, device="cuda", requires_grad=True)
    with pytest.raises(NotImplementedError):
        conv(x, coords, torch.Size([*_level_shapes(g, 4)[1], 8]))


def test_unsorted_pool_input_is_an_error(golden):
    from promptmoge_b200.flex_gemm.ops import build_pool_cache
    g = golden("B_small")
    coords = torch.from_numpy(g["s0_L1_coords"][::-1].copy()).cuda()
    with pytest.raises(ValueError):
        build_pool_cache(coords, _level_shapes(g, 4)[1], (2, 2, 2), (2, 2, 2), (0, 0, 0))


@pytest.mark.parametrize("name,level", [("A_small", 1), ("A_small", 2), ("B_small", 3), ("A_small", 0)])
def test_qat_conv_runs_int8_on_tensor_cores(golden, name, level):
    """A drop-in SubmanifoldConv3d wrapped by the reference's QAT (weight parametrisation + input quantiser pre-hook)
    runs the deployed int8 layer on the tcgen05 kernel: its output is the oracle's dequantised exact int32
    accumulators bit for bit, and within 1e-3 (relative to the output's range) of the fake-quantised fp32 conv."""
    from oracle import refiner as oref
    from promptmoge_b200 import flex_gemm
    from stub_moge import stub_qat
    flex_gemm.install()
    from flex_gemm.nn import SubmanifoldConv3d
    g = golden(name)
    widths = _widths(g)
    C = widths[level]
    coords = torch.from_numpy(g[f"s0_L{level}_coords"]).cuda()
    shape = torch.Size(list(_level_shapes(g, len(widths))[level]) + [C])
    torch.manual_seed(level)
    conv = SubmanifoldConv3d(C, C, 3).cuda().eval()
    x = torch.randn(coords.shape[0], C, device="cuda") * 2.0
    with torch.no_grad():
        y_float, cache = conv(x, coords, shape)                        # no QAT: the fp32 kernel
        aq = stub_qat(conv, clip=5.0)
        y_int8, _ = conv(x, coords, shape, neighbor_cache=cache)       # QAT: the int8 tensor-core kernel
        fq_x = aq(x)
        y_fq, _ = flex_gemm.ops.submanifold_conv(fq_x, coords, shape, conv.weight, conv.bias, neighbor_cache=cache)
    del y_float
    # exact: dequant(oracle int32 accumulators of the quantised input and weight)
    s_a = np.float32(np.float32(5.0) / np.float32(127.0))
    q = np.clip(np.rint(x.cpu().numpy() / s_a), -127, 127).astype(np.int8)
    qw, sw = oref.quant_weight(conv.parametrizations.weight.original.detach().cpu().numpy())
    acc = oref.conv_acc(q, g[f"s0_L{level}_nmap"], qw)
    want = oref.dequant(acc.astype(np.int64), s_a, sw, conv.bias.detach().cpu().numpy())
    np.testing.assert_array_equal(y_int8.cpu().numpy(), want)
    ref = y_fq.cpu().numpy()
    assert np.abs(y_int8.cpu().numpy() - ref).max() <= 1e-3 * np.abs(ref).max()
