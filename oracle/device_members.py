"""The kv tolerance contract with a device member -- TEST INFRASTRUCTURE.

The reference's tolerance for kv_attention floors on four fp32 members
(kernelverify/schemas/native_ops.py:362-394) whose arithmetic is the
dequant-domain numpy port's; its calibration queue names the member a
tensor-core variant would add, the factored integer-domain form
(TODOS.md:230-236). The calibration harness here (oracle/calibrate_k.py,
pre-registered rule in its docstring) scored that form held out and found the
four-member floor unsound at K = 4.0 for it (K 4.38 on one fp32 case of the
independent draw); the rule's first repair -- promote the class's most
demanding member, `factored-serial`, into the floor -- leaves the largest
demand of every other held-out implementation at 2.65, so K = 4.0 stands.

This module is that repaired contract, opt-in: the four shipped members plus
`kv:factored-serial` (integer-domain scores and combine per quantisation
group with serial fp32 sums, the tensor-core kernels' factored form). It can
only widen the tolerance (the floor is a max over a superset of members), so
every verdict the shipped contract passes it passes too; the library's own
parity tests keep the shipped, stricter contract.

Its cost in detection, scored by the harness: none on the rule's own
population (the battery's iid modes, 160 cases); over every battery mode it
lets one caught pair through -- the fp16-score fault on a "near zero" fp32
case (err 4.91e-9 against a tolerance widened from 1.92e-9 to 5.0e-9). A
reference adopting the member trades that canary case for admitting the
factored form.
"""

from __future__ import annotations

import functools

from oracle import kv
from oracle.calibrate_k import factored_serial

KV_DEVICE_MEMBERS = {
    **{name: functools.partial(kv.kv_member, **kw) for name, kw in kv.KV_MEMBERS.items()},
    "kv:factored-serial": factored_serial,
}


def kv_tolerance_device(dtype: str, inputs: dict, ref) -> float:
    """max(4 eps(dtype) max|ref|, K * worst member error) over the shipped
    members and the factored device member, K unchanged at 4.0."""
    return kv.floored_tolerance(kv.base_tol(dtype, ref), kv.K_QUANT,
                                (fn(inputs) for fn in KV_DEVICE_MEMBERS.values()), ref)


def verify_output_device(inputs: dict, candidate, dtype: str = "float16") -> kv.Verdict:
    """The one-step gate under the repaired contract."""
    ref = kv.kv_reference(inputs)
    return kv.judge(candidate, ref, float(kv_tolerance_device(dtype, inputs, ref)))
