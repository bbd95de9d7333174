"""cuDNN C-ABI host logic (no GPU): descriptor validation, output geometry and the
reference's status codes (libraries/dnn/src/cudnn_descriptors.mm, cudnn_ops.mm)."""

import ctypes as C

from muda_b200 import capi
from tests.helpers import Dnn, fptr


def test_handle_and_stream(built):
    L = capi.cudnn()
    assert L.cudnnGetVersion() == 8900
    assert L.cudnnGetErrorString(3) == b"CUDNN_STATUS_BAD_PARAM"
    h = C.c_void_p()
    assert L.cudnnCreate(None) == capi.CUDNN_STATUS_BAD_PARAM
    assert L.cudnnCreate(C.byref(h)) == 0
    s = C.c_void_p(5)
    assert L.cudnnSetStream(h, C.c_void_p(0)) == 0
    assert L.cudnnGetStream(h, C.byref(s)) == 0 and not s.value
    assert L.cudnnDestroy(h) == 0
    assert L.cudnnDestroy(h) == capi.CUDNN_STATUS_BAD_PARAM
    assert L.cudnnSetStream(h, None) == capi.CUDNN_STATUS_BAD_PARAM


def test_tensor_descriptor_rules(built):
    L = capi.cudnn()
    with Dnn() as d:
        t = d.tensor(2, 3, 4, 5, fmt=capi.CUDNN_TENSOR_NHWC)
        v = [C.c_int() for _ in range(9)]
        assert L.cudnnGetTensor4dDescriptor(t, *[C.byref(x) for x in v]) == 0
        assert [x.value for x in v] == [0, 2, 3, 4, 5, 60, 1, 15, 3]
        assert L.cudnnSetTensor4dDescriptor(t, 0, 0, 0, 1, 1, 1) == capi.CUDNN_STATUS_BAD_PARAM
        assert L.cudnnSetTensor4dDescriptor(t, 7, 0, 1, 1, 1, 1) == capi.CUDNN_STATUS_BAD_PARAM
        assert L.cudnnSetTensor4dDescriptor(t, 0, capi.CUDNN_DATA_DOUBLE, 1, 1, 1, 1) == \
            capi.CUDNN_STATUS_NOT_SUPPORTED
        assert L.cudnnSetTensor4dDescriptor(t, 0, 3, 1, 1, 1, 1) == capi.CUDNN_STATUS_BAD_PARAM
        assert L.cudnnSetTensor4dDescriptorEx(t, 0, 1, 2, 2, 2, 8, 4, 2, 0) == \
            capi.CUDNN_STATUS_BAD_PARAM
        # an unconfigured descriptor cannot be read back
        u = C.c_void_p()
        assert L.cudnnCreateTensorDescriptor(C.byref(u)) == 0
        assert L.cudnnGetTensor4dDescriptor(u, *[None] * 9) == capi.CUDNN_STATUS_BAD_PARAM
        assert L.cudnnDestroyTensorDescriptor(u) == 0


def test_conv_output_dim_and_workspace(built):
    L = capi.cudnn()
    with Dnn() as d:
        x = d.tensor(64, 256, 56, 56, fmt=capi.CUDNN_TENSOR_NHWC)
        w = d.filter(256, 256, 3, 3, fmt=capi.CUDNN_TENSOR_NHWC)
        cv = d.conv(pad=(1, 1))
        o = [C.c_int() for _ in range(4)]
        assert L.cudnnGetConvolution2dForwardOutputDim(cv, x, w, *[C.byref(v) for v in o]) == 0
        assert [v.value for v in o] == [64, 256, 56, 56]
        y = d.tensor(64, 256, 56, 56, fmt=capi.CUDNN_TENSOR_NHWC)
        ws = C.c_size_t(7)
        assert L.cudnnGetConvolutionForwardWorkspaceSize(d.h, x, w, cv, y, 0, C.byref(ws)) == 0
        assert ws.value == 0
        bad_y = d.tensor(64, 256, 55, 56)
        assert L.cudnnGetConvolutionForwardWorkspaceSize(d.h, x, w, cv, bad_y, 0, C.byref(ws)) == \
            capi.CUDNN_STATUS_BAD_PARAM
        # strided/dilated geometry: 1 + (7 + 2*2 - (1 + 2*2)) // 2 = 4
        x2 = d.tensor(1, 4, 7, 7)
        w2 = d.filter(8, 2, 3, 3)
        cv2 = d.conv(pad=(2, 2), stride=(2, 2), dil=(2, 2), groups=2)
        assert L.cudnnGetConvolution2dForwardOutputDim(cv2, x2, w2, *[C.byref(v) for v in o]) == 0
        assert [v.value for v in o] == [1, 8, 4, 4]
        g = C.c_int()
        assert L.cudnnGetConvolutionGroupCount(cv2, C.byref(g)) == 0 and g.value == 2
        assert L.cudnnSetConvolutionGroupCount(cv2, 0) == capi.CUDNN_STATUS_BAD_PARAM
        assert L.cudnnSetConvolution2dDescriptor(cv2, -1, 0, 1, 1, 1, 1, 1, 0) == \
            capi.CUDNN_STATUS_BAD_PARAM
        assert L.cudnnSetConvolution2dDescriptor(cv2, 0, 0, 1, 1, 1, 1, 1, 1) == \
            capi.CUDNN_STATUS_NOT_SUPPORTED


def test_forward_argument_errors(built):
    L = capi.cudnn()
    with Dnn() as d:
        x = d.tensor(1, 2, 4, 4)
        w = d.filter(2, 2, 3, 3)
        cv = d.conv(pad=(1, 1))
        y = d.tensor(1, 2, 4, 4)
        p = C.c_void_p(256)
        a, b = fptr(1.0), fptr(0.0)
        assert L.cudnnConvolutionForward(d.h, None, x, p, w, p, cv, 0, None, 0, b, y, p) == \
            capi.CUDNN_STATUS_BAD_PARAM
        assert L.cudnnConvolutionForward(d.h, a, x, None, w, p, cv, 0, None, 0, b, y, p) == \
            capi.CUDNN_STATUS_BAD_PARAM
        # half tensors are valid descriptors but the forward is fp32 (bf16 extension) only
        xh = d.tensor(1, 2, 4, 4, dtype=capi.CUDNN_DATA_HALF)
        wh = d.filter(2, 2, 3, 3, dtype=capi.CUDNN_DATA_HALF)
        yh = d.tensor(1, 2, 4, 4, dtype=capi.CUDNN_DATA_HALF)
        assert L.cudnnConvolutionForward(d.h, a, xh, p, wh, p, cv, 0, None, 0, b, yh, p) == \
            capi.CUDNN_STATUS_NOT_SUPPORTED
        # mismatched shapes
        y3 = d.tensor(1, 3, 4, 4)
        assert L.cudnnSoftmaxForward(d.h, 1, 0, a, x, p, b, y3, p) == capi.CUDNN_STATUS_BAD_PARAM
        # pointers the device cannot address are rejected before any launch
        assert L.cudnnSoftmaxForward(d.h, 1, 0, a, x, p, b, y, p) == capi.CUDNN_STATUS_BAD_PARAM
        stale = C.c_void_p(d.h.value)
    assert L.cudnnSoftmaxForward(stale, 1, 0, fptr(1.0), x, p, fptr(0.0), y, p) == \
        capi.CUDNN_STATUS_BAD_PARAM
