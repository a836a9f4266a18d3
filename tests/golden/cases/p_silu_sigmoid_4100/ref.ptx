.version 8.0
.target sm_89
.address_size 64

.visible .entry k_silu_sigmoid(
        .param .u64 param_x,
        .param .u64 param_out
)
.reqntid 128
{
        .reg .pred      %p<2>;
        .reg .f32       %f<16>;
        .reg .b32       %r<6>;
        .reg .b64       %rd<5>;

        ld.param.u64    %rd1, [param_x];
        cvta.to.global.u64     %rd1, %rd1;
        ld.param.u64    %rd2, [param_out];
        cvta.to.global.u64     %rd2, %rd2;
        mov.u32         %r1, %tid.x;
        mov.u32         %r2, %ntid.x;
        mov.u32         %r3, %ctaid.x;
        mad.lo.s32      %r4, %r3, %r2, %r1;
        mov.u32         %r5, %nctaid.x;
        setp.ge.s32     %p1, %r4, 4100;
        @%p1 bra        SKIP_1;
        mad.wide.s32    %rd3, %r4, 4, %rd1;
        ld.global.nc.f32   %f1, [%rd3];
        neg.f32         %f3, %f1;
        mul.f32         %f4, %f3, 0f3FB8AA3B;
        ex2.approx.ftz.f32 %f5, %f4;
        mov.f32         %f6, 0f3F800000;
        add.f32         %f7, %f6, %f5;
        rcp.rn.f32      %f2, %f7;
        neg.f32         %f9, %f1;
        mul.f32         %f10, %f9, 0f3FB8AA3B;
        ex2.approx.ftz.f32 %f11, %f10;
        mov.f32         %f12, 0f3F800000;
        add.f32         %f13, %f12, %f11;
        rcp.rn.f32      %f14, %f13;
        mul.f32         %f8, %f1, %f14;
        add.f32         %f15, %f2, %f8;
        mad.wide.s32    %rd4, %r4, 4, %rd2;
        st.global.f32   [%rd4], %f15;
SKIP_1:
        ret;
}
