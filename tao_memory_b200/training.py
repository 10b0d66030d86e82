"""Training path of ``tao_attention`` (forward and backward on sm_100a)."""


def tao_attention_train(q, k, v, raw_q, raw_k, fusion_a, fusion_b, alpha, config):
    raise NotImplementedError("training kernels are not built yet")
