"""Test and smoke harness: seeded synthetic decode-step workloads
(``workloads``) and their marshalling into ``MtrSamplerArgs`` for the CPU
oracle and for device launches (``stepargs``).  Not part of the product
package."""
