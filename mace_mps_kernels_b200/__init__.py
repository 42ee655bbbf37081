"""
B200 (sm_100a) CUDA kernels for the two operators that dominate MACE inference, behind a one-call patcher.

Usage: build a float32 MACE model on a CUDA device, then ``report = patch_model(model)``.  The model is modified in
place and the report lists which submodules were swapped and which were left alone (with the reason).

What gets swapped by default:
  * ``interactions.{i}.conv_tp`` -- the per-edge tensor product and its sum over receivers, fused into one kernel
    pair (forward over the receiver CSR, backward over the sender CSR) and switched on through MACE's ``conv_fusion``
    flag;
  * ``products.{i}.symmetric_contractions`` -- evaluated as an explicit per-element polynomial in the node features.
Opt-in extras (not in the reference package): ``edge_features=True`` for the spherical harmonics and the radial basis,
``linears=True`` for the equivariant linears, the skip connections and the radial MLP.  Only first derivatives are
provided, which is what energies, forces, stresses, relaxations and MD need; asking autograd for a second derivative
through these ops raises.
"""
import inspect
import warnings

import torch

from .conv import CudaConvTP, MetalConvTP, conv_supported
from .dense import CudaLinear, CudaSkipTP
from .edge import (CudaRadialEmbedding, CudaSphericalHarmonics, patch_edge_vectors, radial_supported,
                   sh_supported)
from .symmetric import CudaSymmetricContraction, MetalSymmetricContraction, sc_supported

__version__ = '0.1.0'
__all__ = ['patch_model', 'CudaConvTP', 'CudaSymmetricContraction', 'MetalConvTP', 'MetalSymmetricContraction',
           'CudaSphericalHarmonics', 'CudaRadialEmbedding', 'CudaLinear', 'CudaSkipTP']


def _block_has_conv_fusion(blk):
    try:
        return 'conv_fusion' in inspect.getsource(type(blk).forward)
    except (OSError, TypeError):
        return False


def patch_model(model, conv=True, symmetric=True, verbose=True, edge_features=False, linears=False):
    """Swap supported ops for CUDA kernels, in place.  Returns {'patched': [...], 'skipped': [(name, reason)]}.

    Mirrors reference ``__init__.py:34-79``: a float32 model on the accelerator (here CUDA), interaction blocks that
    expose MACE's ``conv_fusion`` path, product blocks without the cuequivariance layout; already-patched blocks are
    left alone (idempotent) and every skip is reported (and warned about when ``verbose``).  Extensions beyond the
    reference, off by default so that the default report is the reference's: ``edge_features=True`` also swaps
    ``spherical_harmonics`` and ``radial_embedding`` and routes the model's ``get_edge_vectors_and_lengths`` to one
    fused launch each way (see ``edge.patch_edge_vectors``); ``linears=True`` swaps every equivariant linear layer,
    the element-indexed skip connections, the radial MLPs and the interactions' ``reshape`` (frozen weights only,
    see ``dense.py``)."""
    p0 = next(model.parameters())
    dev = p0.device
    if dev.type != 'cuda':
        raise RuntimeError(f'model must be on a cuda device (found {dev})')
    if p0.dtype != torch.float32:
        raise RuntimeError('float32 models only')
    patched, skipped = [], []
    with torch.cuda.device(dev):
        if conv:
            for i, blk in enumerate(getattr(model, 'interactions', [])):
                name = f'interactions.{i}.conv_tp'
                if isinstance(getattr(blk, 'conv_tp', None), CudaConvTP):
                    continue
                if hasattr(blk, 'conv_fusion'):
                    skipped.append((name, 'block already uses another fused convolution'))
                    continue
                if not _block_has_conv_fusion(blk):
                    skipped.append((name, f'{type(blk).__name__} has no conv_fusion path'))
                    continue
                ok, why = conv_supported(blk.conv_tp)
                if not ok:
                    skipped.append((name, why))
                    continue
                blk.conv_tp = CudaConvTP(blk.conv_tp)
                blk.conv_fusion = True
                patched.append(name)
        if symmetric:
            for i, prod in enumerate(getattr(model, 'products', [])):
                name = f'products.{i}.symmetric_contractions'
                sc = getattr(prod, 'symmetric_contractions', None)
                if isinstance(sc, CudaSymmetricContraction):
                    continue
                cfg = getattr(prod, 'cueq_config', None)
                if cfg is not None and getattr(cfg, 'enabled', False):
                    skipped.append((name, 'cuequivariance layout'))
                    continue
                ok, why = sc_supported(sc)
                if not ok:
                    skipped.append((name, why))
                    continue
                prod.symmetric_contractions = CudaSymmetricContraction(sc, device=dev)
                patched.append(name)
        if edge_features:
            for name, cls, check in (('spherical_harmonics', CudaSphericalHarmonics, sh_supported),
                                     ('radial_embedding', CudaRadialEmbedding, radial_supported)):
                mod = getattr(model, name, None)
                if isinstance(mod, cls):
                    continue
                ok, why = check(mod)
                if not ok:
                    skipped.append((name, why))
                    continue
                setattr(model, name, cls(mod))
                patched.append(name)
            ok, why = patch_edge_vectors(model)
            (patched.append('get_edge_vectors_and_lengths') if ok
             else skipped.append(('get_edge_vectors_and_lengths', why)))
        if linears:
            from .dense import (CudaFullyConnectedNet, CudaLinear, CudaReshapeIrreps, CudaSkipTP, linear_supported,
                                mlp_supported, reshape_supported, skip_supported)
            for pname, parent in list(model.named_modules()):
                for cname, child in list(parent.named_children()):
                    kind = type(child).__name__
                    if kind == 'Linear' and hasattr(child, 'paths'):
                        cls, (ok, why) = CudaLinear, linear_supported(child)
                    elif kind == 'FullyConnectedTensorProduct' and hasattr(child, 'paths'):
                        cls, (ok, why) = CudaSkipTP, skip_supported(child)
                    elif kind == 'FullyConnectedNet' and hasattr(child, 'hs'):
                        cls, (ok, why) = CudaFullyConnectedNet, mlp_supported(child)
                    elif kind == 'reshape_irreps':
                        cls, (ok, why) = (lambda c: CudaReshapeIrreps(c, device=dev)), reshape_supported(child)
                    else:
                        continue
                    full = f'{pname}.{cname}' if pname else cname
                    if not ok:
                        skipped.append((full, why))
                        continue
                    setattr(parent, cname, cls(child))
                    patched.append(full)
    if verbose:
        for name, why in skipped:
            warnings.warn(f'mace-b200-kernels: kept e3nn for {name}: {why}')
    return dict(patched=patched, skipped=skipped)
