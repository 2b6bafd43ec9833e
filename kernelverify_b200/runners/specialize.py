"""Fill a kernel template's `$NAME` placeholders (source, entry point, name)
and return a finished `KernelSpec` (kernelverify/runners/specialize.py:29-70).

A placeholder the substitutions do not fill raises, and so does a
substitution the template never names -- it is almost always a misspelled
placeholder. CUDA C++ has no `$` in identifiers used by kernels here, so a
placeholder cannot collide with code.
"""

from __future__ import annotations

from string import Template

from kernelverify_b200.runners.spec import KernelSpec, SpecError


def specialize(template: KernelSpec, substitutions: dict) -> KernelSpec:
    texts = {"source": template.source, "entry_point": template.entry_point,
             "name": template.name}
    named: set = set()
    filled = {}
    for where, text in texts.items():
        tmpl = Template(text)
        named.update(tmpl.get_identifiers())
        try:
            filled[where] = tmpl.substitute(substitutions)
        except KeyError as error:
            raise SpecError(f"the template's {where} names ${error.args[0]}, "
                            "which the substitutions do not supply") from error
        except ValueError as error:
            raise SpecError(f"the template's {where} is malformed: {error}") from error
    stray = sorted(set(substitutions) - named)
    if stray:
        raise SpecError(f"substitutions {stray} appear nowhere in the template; "
                        "a misspelled placeholder name looks exactly like this")
    return KernelSpec(source=filled["source"], entry_point=filled["entry_point"],
                      bindings=template.bindings, launch=template.launch, name=filled["name"])
