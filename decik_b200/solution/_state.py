"""State shared by the patches during one training step (solution/_state.py:4-25)."""


class _State:
    def __init__(self):
        # set around the model call by the trainer hook; only then does the packed path run
        self.request = False
        self.stats = None
        # the Packing of the current batch while its forward runs
        self.packing = None
        self.packing_active = False
        # (output, input, weight, eps) of the last RMSNorm on the packed path: the q/v LoRA
        # branch rebuilds its input from the norm's input in backward (solution/attn.py:238)
        self.norm_link = None
        # whether the packed attention runs on the varlen kernels (varlen.patch's switch); the fused
        # attention block calls them directly, so it follows the same switch
        self.varlen_attention = False


STATE = _State()


def on_gpu(tensor):
    """The kernels run on CUDA tensors only; other inputs take the original (unpatched) code."""
    return tensor.is_cuda
