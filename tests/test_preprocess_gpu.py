"""Subsystem 1 parity on the GPU: batched resize + letterbox + normalise
(C-ABI tocr_preprocess_batch_f16/f32) against the C restatement of
preprocess_kernels.cu. fp16 output: within 1 fp16 ulp of the round-to-nearest
of the fp32 oracle. fp32 output: within 2 fp32 ulp."""
import numpy as np
import pytest
import torch

from oracle import preprocess_oracle as po

pytestmark = pytest.mark.gpu


def ulp_dist16(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    def key(x):
        i = x.view(np.int16).astype(np.int32)
        return np.where(i < 0, -(i & 0x7FFF), i)
    return np.abs(key(a) - key(b))


def make_batch(cuda, dims, seed, pitch_pad=0):
    rng = np.random.default_rng(seed)
    imgs, bufs = [], []
    for (h, w) in dims:
        step = w * 3 + pitch_pad
        buf = rng.integers(0, 256, size=(h, step), dtype=np.uint8)
        imgs.append((buf, h, w, step))
        bufs.append(torch.from_numpy(buf).to(cuda))
    return imgs, bufs


def run(tocr, cuda, dims, canvas, out_dtype, seed, limit=("max", 960, 960), pitch_pad=0,
        content=None):
    from turboocr_b200 import kernels as K
    imgs, bufs = make_batch(cuda, dims, seed, pitch_pad)
    if content is None:
        content = [po.det_resize(h, w, *limit) for (h, w) in dims]
    meta = K.PreprocessMeta([b.data_ptr() for b in bufs], [i[3] for i in imgs], dims, content,
                            cuda)
    out = torch.empty(len(dims), 3, canvas[0], canvas[1], dtype=out_dtype, device=cuda)
    K.preprocess_batch(meta, out)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    refs = [po.preprocess_image(buf, content[k], canvas, hw=(h, w), step=step)
            for k, (buf, h, w, step) in enumerate(imgs)]
    return got, np.stack(refs), content


@pytest.mark.parametrize("seed", [0, 1])
def test_fp16_within_one_ulp(tocr, cuda, seed):
    rng = np.random.default_rng(100 + seed)
    dims = [(int(rng.integers(600, 2001)), int(rng.integers(600, 2001))) for _ in range(6)]
    dims += [(640, 700), (960, 960), (300, 1500)]  # <=960 long side: native /32 size
    got, ref, content = run(tocr, cuda, dims, (960, 960), torch.float16, seed)
    d = ulp_dist16(got, ref.astype(np.float16))
    assert d.max() <= 1, d.max()
    # letterbox pad is normalised black
    for k, (ch, cw) in enumerate(content):
        if cw < 960:
            pad = got[k, :, :, cw:]
            exp = ((0.0 - po.DET_MEAN) * po.DET_INV_STD).astype(np.float16)
            assert np.all(pad == exp[:, None, None])


def test_fp32_matches_oracle(tocr, cuda):
    dims = [(777, 1234), (2000, 600), (961, 959)]
    got, ref, _ = run(tocr, cuda, dims, (960, 960), torch.float32, 5)
    np.testing.assert_allclose(got, ref, rtol=0, atol=4e-6)


def test_pitched_rows_and_upscale(tocr, cuda):
    # "min" policy upscales small images; pitch padding exercises src step
    dims = [(40, 90), (33, 47)]
    got, ref, content = run(tocr, cuda, dims, (128, 256), torch.float16, 9,
                            limit=("min", 64, 256), pitch_pad=13)
    assert ulp_dist16(got, ref.astype(np.float16)).max() <= 1


def test_content_larger_edge_cases(tocr, cuda):
    # content not a multiple of 8 and a zero-content image
    dims = [(50, 50), (60, 61)]
    got, ref, _ = run(tocr, cuda, dims, (64, 64), torch.float16, 3,
                      content=[(37, 45), (0, 0)])
    assert ulp_dist16(got, ref.astype(np.float16)).max() <= 1


def test_bit_exact_vs_reference_kernel(tocr, cuda):
    """The reference's own kernel (compiled from its tree) is the tightest
    oracle: the B200 fp32 output must equal it bit for bit, the fp16 output
    must be its round-to-nearest, and the C restatement must agree too."""
    from oracle import ref_kernels as rk
    from turboocr_b200 import kernels as K
    rng = np.random.default_rng(77)
    dims = [(int(rng.integers(600, 2001)), int(rng.integers(600, 2001))) for _ in range(5)]
    dims += [(700, 640), (960, 960)]
    imgs, bufs = make_batch(cuda, dims, 77, pitch_pad=5)
    content = [po.det_resize(h, w, "max", 960, 960) for (h, w) in dims]
    meta = K.PreprocessMeta([b.data_ptr() for b in bufs], [i[3] for i in imgs], dims, content,
                            cuda)
    ref = torch.empty(len(dims), 3, 960, 960, dtype=torch.float32, device=cuda)
    rk.batch_preprocess(meta, ref)
    o32 = torch.empty_like(ref)
    o16 = torch.empty(ref.shape, dtype=torch.float16, device=cuda)
    K.preprocess_batch(meta, o32)
    K.preprocess_batch(meta, o16)
    torch.cuda.synchronize()
    r = ref.cpu().numpy()
    assert np.array_equal(o32.cpu().numpy().view(np.uint32), r.view(np.uint32))
    assert np.array_equal(o16.cpu().numpy().view(np.uint16), r.astype(np.float16).view(np.uint16))
    c = np.stack([po.preprocess_image(buf, content[k], (960, 960), hw=(h, w), step=step)
                  for k, (buf, h, w, step) in enumerate(imgs)])
    mism = int((c.view(np.uint32) != r.view(np.uint32)).sum())
    assert mism == 0, f"C restatement differs from the reference kernel at {mism} values"


def test_config3_full_batch_vs_reference_kernel(tocr, cuda):
    """Config 3 at its full size: 256 images with sides U{600..2000}, the
    det resize policy, one launch; the fp16 canvas must be the
    round-to-nearest of the reference kernel's fp32 canvas everywhere
    (compared on the device)."""
    from oracle import ref_kernels as rk
    from turboocr_b200 import kernels as K
    rng = np.random.default_rng(3)
    dims = [(int(rng.integers(600, 2001)), int(rng.integers(600, 2001))) for _ in range(256)]
    g = torch.Generator(device=cuda).manual_seed(3)
    bufs = [torch.randint(0, 256, (h, w * 3), dtype=torch.uint8, device=cuda, generator=g)
            for (h, w) in dims]
    content = [po.det_resize(h, w, "max", 960, 960) for (h, w) in dims]
    meta = K.PreprocessMeta([b.data_ptr() for b in bufs], [w * 3 for (_, w) in dims], dims,
                            content, cuda)
    ref = torch.empty(256, 3, 960, 960, dtype=torch.float32, device=cuda)
    rk.batch_preprocess(meta, ref)
    o16 = torch.empty(ref.shape, dtype=torch.float16, device=cuda)
    K.preprocess_batch(meta, o16)
    torch.cuda.synchronize()
    assert torch.equal(o16.view(torch.int16), ref.half().view(torch.int16))
