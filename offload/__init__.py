"""Compatibility package: the reference's module paths (`offload.server.main`,
`offload.mobile.main`, `offload.common`, `offload.policies`) mapped onto appcorr_b200."""
