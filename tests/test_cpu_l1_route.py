"""
install_l1(): the name F that a module bound to torch.nn.functional is replaced by a view of it whose l1_loss goes to the library's loss
for float32 CUDA tensors with the mean reduction, and to torch's F.l1_loss for everything else (here: CPU tensors, other reductions);
every other attribute is torch's, and restore() puts the original back. No GPU: the routed calls taken here are torch's.
"""
import sys
import types

import torch
import torch.nn.functional as F

from igs_b200 import autograd as ag


def test_install_l1_routes_only_what_it_computes():
    fake = types.ModuleType("igs_fake_model_cpu")
    fake.F = F
    other = types.ModuleType("igs_fake_other_cpu")
    other.F = "not torch.nn.functional"
    sys.modules["igs_fake_model_cpu"], sys.modules["igs_fake_other_cpu"] = fake, other
    try:
        replaced = ag.install_l1("igs_fake_model_cpu", "igs_fake_other_cpu", "igs_no_such_module")
        assert list(replaced) == [("igs_fake_model_cpu", "F")]
        assert fake.F is not F and other.F == "not torch.nn.functional"
        assert fake.F.mse_loss is F.mse_loss and fake.F.softmax is F.softmax
        a, b = torch.rand(3, 5, 7), torch.rand(3, 5, 7)
        assert torch.equal(fake.F.l1_loss(a, b), F.l1_loss(a, b))                              # CPU tensors: torch's
        assert torch.equal(fake.F.l1_loss(a, b, reduction="sum"), F.l1_loss(a, b, reduction="sum"))
        ag.restore(replaced)
        assert fake.F is F
    finally:
        del sys.modules["igs_fake_model_cpu"], sys.modules["igs_fake_other_cpu"]
