"""A CPU stand-in for rdna4_sage.cp.KernelBackend built on the oracle (test infrastructure): same buffers
and layouts as the C ABI, arithmetic from oracle/sage_oracle.py."""
import numpy as np
import torch

from oracle import sage_oracle as O


class OracleBackend:
    def qk_row_bytes(self, D):
        return 64 if D == 64 else (256 if D == 256 else 128)

    def v_amax(self, v, vs):
        vs.copy_(torch.from_numpy(O.v_amax(v.float().numpy())))

    def quant_q(self, q, fold, q8, qs):
        qn = q.float().numpy()
        c8, cs = O.quant_q(qn)
        if fold != 1.0:
            cs = (cs * np.float32(fold)).astype(np.float32)
        D = qn.shape[-1]
        q8.zero_()
        q8[..., :D] = torch.from_numpy(np.ascontiguousarray(c8.transpose(0, 2, 1, 3)))
        qs.copy_(torch.from_numpy(cs))

    def quant_kv(self, k, v, vs, k8, ks, v8t):
        k8c, ksc, v8c, _ = O.quant_kv(k.float().numpy(), v.float().numpy(), vs.numpy())
        D = k.shape[-1]
        k8.zero_()
        k8[..., :D] = torch.from_numpy(np.ascontiguousarray(k8c.transpose(0, 2, 1, 3)))
        ks.copy_(torch.from_numpy(ksc))
        v8t.copy_(torch.from_numpy(np.ascontiguousarray(v8c.transpose(0, 2, 3, 1))))

    def attn(self, q8, qs, k8, ks, v8t, vs, out, H, Hkv, Sq, Skv, D, causal=False, q_row0=0):
        B = out.shape[0]
        g = H // Hkv
        q8n, qsn, k8n, ksn, v8n, vsn = (t.numpy() for t in (q8, qs, k8, ks, v8t, vs))
        res = np.zeros((B, Sq, H, D), np.float32)
        for b in range(B):
            for h in range(H):
                hk = h // g
                o, _ = O.attention_rows(q8n[b, h, :, :D], qsn[b, h], k8n[b, hk, :, :D], ksn[b, hk],
                                        np.ascontiguousarray(v8n[b, hk].T), vsn[b, hk], np.arange(Sq), Sq, Skv,
                                        causal, block_n=32, row0=q_row0)
                res[b, :, h] = o
        out.copy_(torch.from_numpy(res).to(out.dtype))

    def attn_chunked(self, q8, qs, k8, ks, v8t, vs, out, H, Hkv, Sq, Skv, D, causal, q_row0):
        # the chunked layout reassembled to the plain one ([n, B, Hkv, chunk, ...] -> [B, Hkv, n * chunk, ...])
        n, B, _, chunk = k8.shape[:4]
        k8f = k8.permute(1, 2, 0, 3, 4).reshape(B, Hkv, n * chunk, -1)
        ksf = ks.permute(1, 2, 0, 3).reshape(B, Hkv, -1)
        v8f = v8t.permute(1, 2, 3, 0, 4).reshape(B, Hkv, D, n * chunk)
        self.attn(q8, qs, k8f, ksf, v8f, vs, out, H, Hkv, Sq, Skv, D, causal=causal, q_row0=q_row0)
