"""FP32 PyTorch references of canonical SPAN x2, classic IFNet and RIFE 4.2x, for parity at full frame sizes
(test aid only: the tests and bench.py's output check use them, the product never does).

The numpy oracle (oracle/nets.py, pinned to the reference's interpreter) needs minutes for one
1920x1080 SPAN frame and for a 4K IFNet pair, so full-size checks compare against these
restatements of the same networks in torch FP32 instead (cuDNN / CPU convolutions with TF32 off).
tests/test_torch_ref.py pins them to the numpy oracle on the CPU; the GPU tests pin them again on a
crop before they use them."""
from __future__ import annotations

import numpy as np

import seeded


def _fp32_mode():
    import torch
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.deterministic = True


def span_forward(x, p, device="cuda"):
    """nets.span_forward (no quantisation) in torch FP32: x [n,3,h,w] numpy or torch -> numpy
    [n,3,2h,2w], frame by frame to bound device memory."""
    import torch
    import torch.nn.functional as F
    _fp32_mode()
    w = {k: torch.from_numpy(np.ascontiguousarray(v, np.float32)).to(device) for k, v in p.items()}
    xs = torch.as_tensor(np.asarray(x, np.float32)) if not isinstance(x, torch.Tensor) else x.float()
    outs = []
    with torch.no_grad():
        for i in range(xs.shape[0]):
            xi = xs[i:i + 1].to(device)
            s0 = F.conv2d(xi, w["conv_1.w"], w["conv_1.b"], padding=1)
            xb = s0
            first = last_act = None
            for b in range(seeded.SPAN_BLOCKS):
                a1 = F.silu(F.conv2d(xb, w[f"block{b}.c1.w"], w[f"block{b}.c1.b"], padding=1))
                a2 = F.silu(F.conv2d(a1, w[f"block{b}.c2.w"], w[f"block{b}.c2.b"], padding=1))
                c3 = F.conv2d(a2, w[f"block{b}.c3.w"], w[f"block{b}.c3.b"], padding=1)
                xb = (c3 + xb) * (torch.sigmoid(c3) - 0.5)
                if b == 0:
                    first = xb
                if b == seeded.SPAN_BLOCKS - 1:
                    last_act = a1
            cat = torch.cat([s0, xb, first, last_act], dim=1)
            fused = F.conv2d(cat, w["conv_cat.w"], w["conv_cat.b"])
            up = F.conv2d(fused, w["upsampler.w"], w["upsampler.b"], padding=1)
            outs.append(F.pixel_shuffle(up, 2).cpu())
            del s0, xb, first, last_act, cat, fused, up
    return torch.cat(outs).numpy()


def _warp(img, fx, fy):
    """Backward warp of img [1,c,h,w] by flow planes fx, fy [h,w] with the reference's tap rule
    (warp_lib.cuh:45-58): ix = x + fx in FP32, NaN to 0, clamped to [0, w - 1], x0 = trunc(ix),
    x1 = min(x0 + 1, w - 1), weight ix - x0; the same along y; whole-plane window."""
    import torch
    _, c, h, w = img.shape
    xs = torch.arange(w, dtype=torch.float32, device=img.device)[None, :]
    ys = torch.arange(h, dtype=torch.float32, device=img.device)[:, None]
    ix = torch.nan_to_num(xs + fx, nan=0.0).clamp(0, w - 1)
    iy = torch.nan_to_num(ys + fy, nan=0.0).clamp(0, h - 1)
    x0, y0 = ix.to(torch.int64), iy.to(torch.int64)
    x1, y1 = (x0 + 1).clamp(max=w - 1), (y0 + 1).clamp(max=h - 1)
    wx, wy = ix - x0.float(), iy - y0.float()
    flat = img.reshape(c, h * w)

    def at(yy, xx):
        return flat[:, (yy * w + xx).reshape(-1)].reshape(c, h, w)

    top = at(y0, x0) * (1 - wx) + at(y0, x1) * wx
    bot = at(y1, x0) * (1 - wx) + at(y1, x1) * wx
    return (top * (1 - wy) + bot * wy)[None]


def ifnet_forward(img0, img1, timestep, p, device="cuda", return_flow=False):
    """nets.ifnet_forward in torch FP32 on one pair img0, img1 [1,3,h,w] (h, w multiples of 32) ->
    numpy [1,3,h,w] (and the flow [1,4,h,w] and pre-sigmoid mask [1,1,h,w] with return_flow)."""
    import torch
    import torch.nn.functional as F
    _fp32_mode()
    w = {k: torch.from_numpy(np.ascontiguousarray(v, np.float32)).to(device) for k, v in p.items()}
    a = torch.as_tensor(np.asarray(img0, np.float32)).to(device)
    b = torch.as_tensor(np.asarray(img1, np.float32)).to(device)
    _, _, h, wd = a.shape
    t = torch.full((1, 1, h, wd), float(timestep), device=device)

    def resize(x, hh, ww):
        return F.interpolate(x, size=(hh, ww), mode="bilinear", align_corners=False)

    def block(x, flow, scale, k):
        if scale != 1:
            x = resize(x, h // scale, wd // scale)
        if flow is not None:
            f = resize(flow, h // scale, wd // scale) if scale != 1 else flow
            x = torch.cat([x, f * (1.0 / scale)], 1)
        y = F.prelu(F.conv2d(x, w[f"b{k}.conv0a.w"], w[f"b{k}.conv0a.b"], stride=2, padding=1), w[f"b{k}.conv0a.slope"])
        y = F.prelu(F.conv2d(y, w[f"b{k}.conv0b.w"], w[f"b{k}.conv0b.b"], stride=2, padding=1), w[f"b{k}.conv0b.slope"])
        for j in range(seeded.IFNET_RES):
            r = F.conv2d(y, w[f"b{k}.res{j}.w"], w[f"b{k}.res{j}.b"], padding=1)
            y = F.prelu(r + y, w[f"b{k}.res{j}.slope"])
        tmp = F.conv_transpose2d(y, w[f"b{k}.last.w"], w[f"b{k}.last.b"], stride=2, padding=1)
        tmp = resize(tmp, h, wd)
        return tmp[:, :4] * float(scale * 2), tmp[:, 4:5]

    with torch.no_grad():
        flow = mask = None
        w0, w1 = a, b
        for k, s in enumerate(seeded.IFNET_SCALES):
            if k == 0:
                flow, mask = block(torch.cat([a, b, t], 1), None, s, k)
            else:
                fd, md = block(torch.cat([w0, w1, t, mask], 1), flow, s, k)
                flow = flow + fd
                mask = mask + md
            w0 = _warp(a, flow[0, 0], flow[0, 1])
            w1 = _warp(b, flow[0, 2], flow[0, 3])
        m = torch.sigmoid(mask)
        out = w0 * m + w1 * (1 - m)
    if return_flow:
        return out.cpu().numpy(), flow.cpu().numpy(), mask.cpu().numpy()
    return out.cpu().numpy()


def rife42_forward(img0, img1, timestep, flat, device="cuda"):
    """RIFE 4.2x (oracle/ref_graphs.cpp kref_rife42_forward) in torch FP32 on one pair img0, img1
    [1,3,h,w] (h, w multiples of 4 * max d): (image [1,3,h,w], flow [1,4,h,w], sigmoid(mask)
    [1,1,h,w]) as numpy. flat: the C ABI's parameter array (12 plan floats first)."""
    import torch
    import torch.nn.functional as F
    _fp32_mode()
    flat = np.asarray(flat, np.float32)
    blocks = int(flat[0])
    plan = (blocks, tuple(int(v) for v in flat[1:1 + blocks]), tuple(int(v) for v in flat[6:6 + blocks]))
    p = seeded.unflatten(flat[seeded.RIFE_PLAN_FLOATS:], seeded.rife_param_shapes(plan))
    w = {k: torch.from_numpy(np.ascontiguousarray(v, np.float32)).to(device) for k, v in p.items()}
    a = torch.as_tensor(np.asarray(img0, np.float32)).to(device)
    b = torch.as_tensor(np.asarray(img1, np.float32)).to(device)
    _, _, h, wd = a.shape
    t = torch.full((1, 1, h, wd), float(timestep), device=device)

    def resize(x, hh, ww):
        return F.interpolate(x, size=(hh, ww), mode="bilinear", align_corners=False)

    def act(x, name):
        return F.prelu(x, w[name + ".slope"])

    def encode(x):
        e = act(F.conv2d(x, w["enc.cnn0.w"], w["enc.cnn0.b"], stride=2, padding=1), "enc.cnn0")
        e = act(F.conv2d(e, w["enc.cnn1.w"], w["enc.cnn1.b"], padding=1), "enc.cnn1")
        e = act(F.conv2d(e, w["enc.cnn2.w"], w["enc.cnn2.b"], padding=1), "enc.cnn2")
        return F.conv_transpose2d(e, w["enc.cnn3.w"], w["enc.cnn3.b"], stride=2, padding=1)

    def block(x, flow, d, k):
        if d != 1:
            x = resize(x, h // d, wd // d)
        if flow is not None:
            f = resize(flow, h // d, wd // d) if d != 1 else flow
            x = torch.cat([x, f * (1.0 / d)], 1)
        y = act(F.conv2d(x, w[f"b{k}.conv0a.w"], w[f"b{k}.conv0a.b"], stride=2, padding=1), f"b{k}.conv0a")
        y = act(F.conv2d(y, w[f"b{k}.conv0b.w"], w[f"b{k}.conv0b.b"], stride=2, padding=1), f"b{k}.conv0b")
        for j in range(seeded.IFNET_RES):
            r = F.conv2d(y, w[f"b{k}.res{j}.w"], w[f"b{k}.res{j}.b"], padding=1)
            y = act(r * w[f"b{k}.res{j}.beta"][None, :, None, None] + y, f"b{k}.res{j}")
        tmp = F.pixel_shuffle(F.conv_transpose2d(y, w[f"b{k}.last.w"], w[f"b{k}.last.b"], stride=2, padding=1), 2)
        if d != 1:
            tmp = resize(tmp, h, wd)
        return tmp[:, :4] * float(d), tmp[:, 4:5], tmp[:, 5:13]

    with torch.no_grad():
        fa, fb = encode(a), encode(b)
        flow = mask = feat = None
        w0, w1, wf0, wf1 = a, b, fa, fb
        for k in range(blocks):
            d = plan[1][k]
            if k == 0:
                flow, mask, feat = block(torch.cat([a, b, fa, fb, t], 1), None, d, k)
            else:
                fd, mask, feat = block(torch.cat([w0, w1, wf0, wf1, t, mask, feat], 1), flow, d, k)
                flow = flow + fd
            w0 = _warp(a, flow[0, 0], flow[0, 1])
            w1 = _warp(b, flow[0, 2], flow[0, 3])
            if k + 1 < blocks:
                wf0 = _warp(fa, flow[0, 0], flow[0, 1])
                wf1 = _warp(fb, flow[0, 2], flow[0, 3])
        m = torch.sigmoid(mask)
        out = w0 * m + w1 * (1 - m)
    return out.cpu().numpy(), flow.cpu().numpy(), m.cpu().numpy()
