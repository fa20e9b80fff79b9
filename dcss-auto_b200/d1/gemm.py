"""Dense layers of the policy: y = relu(x @ w^T + b), bf16 in/out, fp32 accumulate."""
import torch


def linear_relu(x, w, b):
    return torch.nn.functional.linear(x, w, b.to(torch.bfloat16)).relu_()
