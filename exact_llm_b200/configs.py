"""Model architectures of the benchmark configurations (reference config-dict keys,
exact_llm.py:227-230), plus ``lin``: "group" (group-128 GQLin layers) or "channel" (QLin)."""

ARCHS = {
    "qwen2.5-0.5b": dict(D=896, H=14, KV=2, hd=64, I=4864, V=151936, NL=24, theta=1e6, tie=True, lin="group"),
    "qwen2.5-7b": dict(D=3584, H=28, KV=4, hd=128, I=18944, V=152064, NL=28, theta=1e6, tie=False, lin="group"),
    "qwen2.5-14b": dict(D=5120, H=40, KV=8, hd=128, I=13824, V=152064, NL=48, theta=1e6, tie=False, lin="group"),
    "qwen1.5-moe-a2.7b": dict(D=2048, H=16, KV=16, hd=128, I=1408, V=151936, NL=24, theta=1e6, tie=False,
                              lin="channel", NE=60, TOPK=4, MI=1408, SI=5632),
}


def arch(name, **over):
    c = dict(ARCHS[name])
    c.update(over)
    return c
