"""The operator list of ntops.torch (src/ntops/torch/__init__.py:1-115) restricted to the LLM hot
path; every operator has the reference's signature."""

from ntops_b200.torch.abs import abs
from ntops_b200.torch.add import add
from ntops_b200.torch.addmm import addmm
from ntops_b200.torch.bitwise_and import bitwise_and
from ntops_b200.torch.bitwise_not import bitwise_not
from ntops_b200.torch.bitwise_or import bitwise_or
from ntops_b200.torch.bmm import bmm
from ntops_b200.torch.clamp import clamp
from ntops_b200.torch.conv2d import conv2d
from ntops_b200.torch.copysign import copysign
from ntops_b200.torch.cos import cos
from ntops_b200.torch.div import div
from ntops_b200.torch.dropout import dropout
from ntops_b200.torch.eq import eq
from ntops_b200.torch.exp import exp
from ntops_b200.torch.frac import frac
from ntops_b200.torch.ge import ge
from ntops_b200.torch.gelu import gelu
from ntops_b200.torch.gt import gt
from ntops_b200.torch.isinf import isinf
from ntops_b200.torch.isnan import isnan
from ntops_b200.torch.layer_norm import layer_norm
from ntops_b200.torch.lcm import lcm
from ntops_b200.torch.le import le
from ntops_b200.torch.lgamma import lgamma
from ntops_b200.torch.lt import lt
from ntops_b200.torch.matmul import matmul
from ntops_b200.torch.mm import mm
from ntops_b200.torch.mul import mul
from ntops_b200.torch.ne import ne
from ntops_b200.torch.neg import neg
from ntops_b200.torch.nextafter import nextafter
from ntops_b200.torch.pow import pow
from ntops_b200.torch.rad2deg import rad2deg
from ntops_b200.torch.relu import relu
from ntops_b200.torch.rms_norm import rms_norm
from ntops_b200.torch.rotary_position_embedding import rotary_position_embedding
from ntops_b200.torch.rsqrt import rsqrt
from ntops_b200.torch.scaled_dot_product_attention import scaled_dot_product_attention
from ntops_b200.torch.sigmoid import sigmoid
from ntops_b200.torch.silu import silu
from ntops_b200.torch.sin import sin
from ntops_b200.torch.softmax import softmax
from ntops_b200.torch.sub import sub
from ntops_b200.torch.tanh import tanh

__all__ = [
    "abs",
    "add",
    "addmm",
    "bitwise_and",
    "bitwise_not",
    "bitwise_or",
    "bmm",
    "clamp",
    "conv2d",
    "copysign",
    "cos",
    "div",
    "dropout",
    "eq",
    "exp",
    "frac",
    "ge",
    "gelu",
    "gt",
    "isinf",
    "isnan",
    "layer_norm",
    "lcm",
    "le",
    "lgamma",
    "lt",
    "matmul",
    "mm",
    "mul",
    "ne",
    "neg",
    "nextafter",
    "pow",
    "rad2deg",
    "relu",
    "rms_norm",
    "rotary_position_embedding",
    "rsqrt",
    "scaled_dot_product_attention",
    "sigmoid",
    "silu",
    "sin",
    "softmax",
    "sub",
    "tanh",
]
