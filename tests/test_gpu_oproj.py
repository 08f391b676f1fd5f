"""GPU tests of the output projection fused with its reduce-scatter
(vk_oproj_*): the `wo` matmul after attention, checked against the oracle's
restatement of the reference's launch_matmul (cuda/matmul.cu:42-103) on the
same fp16 inputs widened to fp32.  Outputs are fp16 under the attention
tolerance.  The two-GPU reduce-scatter is in test_gpu_multi.py; here one rank,
repeated runs, the weight packing and a wait that must time out."""
import time

import numpy as np
import pytest
import torch

import oracle
from tests.helpers import assert_close_attn

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def vk(cuda_ok):
    import vulcan_b200
    vulcan_b200.load()
    return vulcan_b200


def _inputs(rng, tokens, k, n):
    x = (rng.standard_normal((tokens, k)) * 0.5).astype(np.float16)
    w = (rng.standard_normal((k, n)) * 0.02).astype(np.float16)  # wo rows [k, n]
    return x, w


@pytest.mark.parametrize("tokens,k,n", [(1, 128, 256), (16, 1024, 1024), (64, 1024, 8192), (100, 4096, 2048),
                                        (256, 512, 1024), (48, 192, 384)])
def test_oproj_one_rank_matches_oracle(vk, tokens, k, n):
    rng = np.random.default_rng(tokens * 7 + k + n)
    x, w = _inputs(rng, tokens, k, n)
    op = vk.OutputProjection(0, 1, max(tokens, 64), k, n)
    wp = op.pack_weight(torch.from_numpy(w.astype(np.float32)).cuda())  # the reference's fp32 wo rows
    y = op.run(torch.from_numpy(x).cuda(), wp)
    torch.cuda.synchronize()
    op.check()
    ref = oracle.matmul(x.astype(np.float32), w.astype(np.float32))
    assert_close_attn(y.float().cpu().numpy(), ref, "oproj tokens %d k %d n %d (splits %d)" % (tokens, k, n, op.splits))
    op.close()


def test_oproj_strided_inputs_and_output(vk):
    """x given as a column slice of the full attention output (a rank's heads),
    the weight packed from a column slice of the nn.Linear [out, in] weight,
    y written into a wider buffer."""
    rng = np.random.default_rng(5)
    tokens, K, k, n = 24, 1024, 256, 512
    xf, wf = _inputs(rng, tokens, K, n)
    r0 = 512  # this rank's rows of wo / columns of x
    op = vk.OutputProjection(0, 1, 64, k, n)
    xd = torch.from_numpy(xf).cuda()
    wtd = torch.from_numpy(np.ascontiguousarray(wf.T)).cuda()  # [n, K]
    ybig = torch.zeros(tokens, n + 64, dtype=torch.float16, device="cuda")
    op.run(xd[:, r0:r0 + k], op.pack_weight_t16(wtd[:, r0:r0 + k]), y=ybig[:, :n])
    torch.cuda.synchronize()
    ref = oracle.matmul(xf[:, r0:r0 + k].astype(np.float32), wf[r0:r0 + k].astype(np.float32))
    assert_close_attn(ybig[:, :n].float().cpu().numpy(), ref, "strided")
    assert torch.count_nonzero(ybig[:, n:]).item() == 0
    op.close()


def test_oproj_repeated_runs_bit_identical(vk):
    """Runs alternate receive slots and flag values; the sum order is fixed, so
    every run gives the same bits."""
    rng = np.random.default_rng(6)
    x, w = _inputs(rng, 64, 2048, 4096)
    op = vk.OutputProjection(0, 1, 64, 2048, 4096)
    xd, wtd = torch.from_numpy(x).cuda(), op.pack_weight_t16(torch.from_numpy(np.ascontiguousarray(w.T)).cuda())
    first = op.run(xd, wtd).clone()
    for _ in range(5):
        assert torch.equal(op.run(xd, wtd), first)
    op.check()
    op.close()


def _packed_reference(w16):
    """The packed layout restated on the host: 16 KiB blocks [n/128][k/64] of
    128 rows (features) x 64 k, 16-byte chunk c of row r at c ^ (r % 8)."""
    k, n = w16.shape
    out = np.zeros((n // 128, k // 64, 128, 8, 8), np.float16)
    wt = w16.T.reshape(n // 128, 128, k // 64, 8, 8)  # [tile, r, kb, chunk, e]
    for r in range(128):
        for c in range(8):
            out[:, :, r, c ^ (r & 7), :] = wt[:, r, :, c, :]
    return out.reshape(-1).view(np.uint8)


def test_oproj_pack_weight_layouts(vk):
    """Both packers produce the same bytes, equal to the layout restated here."""
    rng = np.random.default_rng(7)
    w = (rng.standard_normal((192, 256)) * 0.02).astype(np.float32)  # [k_rows, n]
    a = vk.OutputProjection.pack_weight(torch.from_numpy(w).cuda())
    b = vk.OutputProjection.pack_weight_t16(torch.from_numpy(np.ascontiguousarray(w.T.astype(np.float16))).cuda())
    torch.cuda.synchronize()
    want = _packed_reference(w.astype(np.float16))
    assert np.array_equal(a.cpu().numpy(), want)
    assert np.array_equal(b.cpu().numpy(), want)


def test_oproj_rejects_bad_arguments(vk):
    with pytest.raises(vk.VKError):
        vk.OutputProjection(0, 1, 64, 100, 1024)      # k_local not a multiple of 64
    with pytest.raises(vk.VKError):
        vk.OutputProjection(0, 2, 64, 128, 384)       # n_out not a multiple of 128 * world
    with pytest.raises(vk.VKError):
        vk.OutputProjection(0, 1, 300, 128, 256)      # more than 256 tokens
    op = vk.OutputProjection(0, 1, 32, 128, 256)
    x = torch.zeros(33, 128, dtype=torch.float16, device="cuda")
    wp = op.pack_weight_t16(torch.zeros(256, 128, dtype=torch.float16, device="cuda"))
    with pytest.raises(vk.VKError):
        op.run(x, wp)                                 # more tokens than max_tokens
    with pytest.raises(ValueError):
        op.run(x[:8], wp[:100])                       # not a packed weight of this shape
    op.close()


def test_oproj_wait_times_out(vk):
    """Rank 0 of two, with rank 1 a projection of this process on the same GPU
    that never runs: rank 0's tiles wait for rank 1's contributions, the bounded
    wait gives up after about 1 s, and the host reads VK_TIMEOUT once.  Only one
    kernel waits, on a flag that nothing sets.  A one-rank projection then runs
    normally on the same device."""
    rng = np.random.default_rng(8)
    x, w = _inputs(rng, 16, 256, 512)
    a, b = vk.OutputProjection(0, 2, 16, 256, 512), vk.OutputProjection(1, 2, 16, 256, 512)
    a.import_local(1, b)
    b.import_local(0, a)
    xd, wtd = torch.from_numpy(x).cuda(), a.pack_weight_t16(torch.from_numpy(np.ascontiguousarray(w.T)).cuda())
    torch.cuda.synchronize()
    t0 = time.monotonic()
    a.run(xd, wtd)
    torch.cuda.synchronize()
    waited = time.monotonic() - t0
    assert 0.9 < waited < 10.0, "the wait must give up after its 1 s bound (took %.2f s)" % waited
    with pytest.raises(vk.VKError) as e:
        a.check()
    assert e.value.status == 4  # VK_TIMEOUT
    a.check()  # cleared
    a.close()
    b.close()
    one = vk.OutputProjection(0, 1, 16, 256, 512)
    y = one.run(xd, wtd)
    torch.cuda.synchronize()
    one.check()
    assert_close_attn(y.float().cpu().numpy(), oracle.matmul(x.astype(np.float32), w.astype(np.float32)), "after")
    one.close()
