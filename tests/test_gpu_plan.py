"""The packed prefill plan built on the device (vk_prefill_plan) equals the host construction of
viktor/engine.py:145-159 (``prefill_plan``, itself checked against the reference's torch code on CPU), and a
caller whose sizes disagree with the lengths gets a range error and untouched outputs."""

import numpy as np
import pytest
import torch

from viktor_b200.engine import prefill_plan

pytestmark = pytest.mark.gpu


def device_plan(lens, row0, pos_scale, total=None):
    from viktor_b200._lib import call
    dev = torch.device("cuda")
    n, frames = len(lens), int(sum(lens))
    total = frames + n if total is None else total
    fill = dict(device=dev)
    out = dict(cu=torch.full((n + 1,), -7, dtype=torch.int32, **fill),
               frame_idx=torch.full((max(frames, 1),), -7, dtype=torch.int32, **fill),
               last=torch.full((n,), -7, dtype=torch.int64, **fill),
               pos=torch.full((max(total, 1),), -7, dtype=torch.int32, **fill),
               seq=torch.full((max(total, 1),), -7, dtype=torch.int32, **fill),
               rpos=torch.full((max(total, 1),), -7, dtype=torch.int32, **fill),
               lengths=torch.full((n,), -7, dtype=torch.int32, **fill))
    lens_d = torch.tensor(lens, dtype=torch.int32, device=dev)
    call("vk_prefill_plan", lens_d.data_ptr(), n, row0, pos_scale, total, out["cu"].data_ptr(),
         out["frame_idx"].data_ptr(), out["last"].data_ptr(), out["pos"].data_ptr(), out["seq"].data_ptr(),
         None if pos_scale == 1 else out["rpos"].data_ptr(), out["lengths"].data_ptr(),
         torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return {k: v.cpu().numpy() for k, v in out.items()}


CASES = [([5, 0, 17, 3], 0, 1), ([2048] * 128, 0, 1), ([2048, 128, 1], 128, 1), ([9, 30], 2, 4), ([0], 5, 1),
         (list(np.random.default_rng(0).integers(0, 40, 4096)), 0, 2), ([1], 0, 1)]


@pytest.mark.parametrize("lens,row0,pos_scale", CASES)
def test_device_plan_equals_host_plan(lens, row0, pos_scale):
    from viktor_b200._lib import check_device_errors
    lens = [int(v) for v in lens]
    ref = prefill_plan(lens, row0, pos_scale)
    got = device_plan(lens, row0, pos_scale)
    check_device_errors()
    total, frames = ref["total"], ref["frames"]
    assert np.array_equal(got["cu"], ref["cu"])
    assert np.array_equal(got["frame_idx"][:frames], ref["frame_idx"])
    assert np.array_equal(got["last"], ref["last"])
    assert np.array_equal(got["pos"][:total], ref["pos"])
    assert np.array_equal(got["seq"][:total], ref["seq"])
    assert np.array_equal(got["lengths"], ref["lengths"])
    if pos_scale != 1:
        assert np.array_equal(got["rpos"][:total], ref["rpos"])


def test_device_plan_rejects_inconsistent_sizes():
    from viktor_b200._lib import DEVERR, read_device_errors
    read_device_errors(clear=True)
    got = device_plan([5, 7], 0, 1, total=15)  # 5 + 7 + 2 = 14
    bits = read_device_errors(clear=True)
    assert bits & next(b for b, m in DEVERR.items() if "range" in m or "bound" in m.lower())
    assert (got["cu"] == -7).all() and (got["pos"] == -7).all() and (got["frame_idx"] == -7).all()
